"""SGLang ``pp_group`` backed by the Connex step protocol (external, elastic PP;
communication side only, reference ``connex/adapters/sglang/pp_group.py``).

SGLang's scheduler reaches its pipeline neighbours only through
``scheduler.pp_group`` (a ``GroupCoordinator``): ``send_tensor_dict`` /
``recv_tensor_dict`` tagged ``"__msg_type__": "proxy"`` (hidden states going
forward) or ``"output"`` (sampled tokens coming back), plus the rank
properties.  :class:`ConnexPPGroup` serves that surface over a step transport
(:class:`connex.pp.endpoint.PipelineEndpoint`, or the in-process fake of
``connex.pp.testing``) in the external topology:

* stage 0 runs the only scheduler.  A ``proxy`` send starts a step through
  :class:`connex.pp.link.Stage0Link` (new correlation id, ``cx_ctx`` and
  finished ids attached); a receive returns the ``output`` of the oldest
  outstanding step (SGLang consumes microbatch results in launch order).
  Re-sends after a failover and the ``reprefill`` hook are Stage0Link's.
* stages 1.. are passive executors.  A receive returns the next step's
  ``proxy`` dict after the KV-ownership check: rows whose KV this stage does
  not hold are released and listed under :data:`MISSING_HERE` (the engine
  must not cache them).  The next send answers that step: forwarded to the
  next stage, or from the last stage as the ``output`` back to stage 0, with
  the missing rows merged into ``cx_missing``.

The engine side (one scheduler on stage 0, stateless executors that load
only their layers, per-request KV accounting, re-prefill) is SGLang's.
"""
from __future__ import annotations

import logging
from collections import deque
from typing import Any, Callable, Optional, Sequence

from connex.pp.handover import CX_CTX, CX_MISSING, FINISHED, REQUEST_IDS, find_missing, merge_missing
from connex.pp.link import Stage0Link

MSG_TYPE = "__msg_type__"
MISSING_HERE = "__cx_missing_here__"     # stages 1..: rows this stage has no KV for
REPREFILLED = "__cx_reprefilled__"       # stage 0: rows the engine must recompute

_log = logging.getLogger("connex.adapters.sglang")


class _Completed:
    """SGLang's P2P work handle (``.work.wait()``); a Connex send has been
    handed to the endpoint when it returns."""

    class _Work:
        def wait(self):
            return True

        def is_completed(self):
            return True

    def __init__(self):
        self.work = self._Work()


class ConnexPPGroup:
    """``GroupCoordinator``-compatible PP group of one external stage.

    ``row_info()`` (stage 0, optional) gives ``(request_ids, num_computed)``
    of the batch being sent (for ``cx_ctx``); ``hooks`` implements
    :class:`connex.pp.hooks.EngineHooks`."""

    def __init__(self, transport, hooks=None, *, row_info: Optional[Callable[[], tuple]] = None,
                 recv_timeout_s: Optional[float] = None, max_attempts: int = 5, log: logging.Logger = _log):
        self.t = transport
        self.hooks = hooks
        self.row_info = row_info
        self.log = log
        self.world_size = transport.num_stages
        self.rank_in_group = transport.stage_idx
        self.ranks = list(range(self.world_size))
        self.device_group = self.cpu_group = None
        self._head = Stage0Link(transport, hooks, recv_timeout_s=recv_timeout_s, max_attempts=max_attempts,
                                log=log) if transport.is_first else None
        self._outstanding: deque = deque()      # stage 0: correlation ids in launch order
        self._answer: deque = deque()           # stages 1..: (reply ctx, received dict)
        self.stats = {"sent": 0, "received": 0, "missing": 0}

    # ---- GroupCoordinator properties -------------------------------------------
    @property
    def is_first_rank(self) -> bool:
        return self.t.is_first

    @property
    def is_last_rank(self) -> bool:
        return self.t.is_last

    @property
    def next_rank(self) -> int:
        return (self.rank_in_group + 1) % self.world_size

    @property
    def prev_rank(self) -> int:
        return (self.rank_in_group - 1) % self.world_size

    def finished(self, request_ids: Sequence) -> None:
        """Stage 0: requests that ended (their KV is freed downstream)."""
        if self._head is not None:
            self._head.finished(request_ids)

    # ---- data path ----------------------------------------------------------------
    def send_tensor_dict(self, tensor_dict: dict, dst: Optional[int] = None, all_gather_group: Any = None,
                         async_send: bool = False):
        """``all_gather_group`` is ignored: one sender per stage sends whole tensors."""
        self.stats["sent"] += 1
        if self.t.is_first:
            rids, ncomp = self.row_info() if self.row_info is not None else (None, None)
            self._outstanding.append(self._head.submit(dict(tensor_dict), rids, ncomp))
            return [_Completed()]
        if not self._answer:
            raise RuntimeError("ConnexPPGroup: a later stage sends only to answer a received step")
        ctx, got = self._answer.popleft()
        out = {k: v for k, v in tensor_dict.items() if k != MISSING_HERE}
        missing = merge_missing(got.get(CX_MISSING), got.get(MISSING_HERE))
        if missing:
            out[CX_MISSING] = missing
        if self.t.is_last:
            out[MSG_TYPE] = "output"
        else:
            for k in (REQUEST_IDS, CX_CTX, FINISHED):
                if k in got:
                    out.setdefault(k, got[k])
        self.t.send_reply(out, ctx)
        return [_Completed()]

    def recv_tensor_dict(self, src: Optional[int] = None, all_gather_group: Any = None) -> dict:
        self.stats["received"] += 1
        if self.t.is_first:
            if not self._outstanding:
                raise RuntimeError("ConnexPPGroup: stage 0 receive without an outstanding step")
            reply = self._head.wait(self._outstanding.popleft())
            reply.setdefault(MSG_TYPE, "output")
            return reply
        td, ctx = None, None
        while td is None:
            td, ctx = self.t.recv_forward()
        rids = td.get(REQUEST_IDS) or []
        if self.hooks is not None:
            live = set(rids)
            ended = [r for r in td.get(FINISHED) or () if r not in live]
            if ended:
                self.hooks.release(ended)
        lacking = find_missing(rids, td.get(CX_CTX), self.hooks.kv_held) if self.hooks is not None else []
        if lacking:
            self.log.warning("stage %s: no KV here for %d of %d request(s)", self.t.stage_idx, len(lacking),
                             len(rids))
            self.hooks.release(lacking)
            self.stats["missing"] += len(lacking)
        td[MISSING_HERE] = lacking
        td.setdefault(MSG_TYPE, "proxy")
        self._answer.append((ctx, td))
        return td

    def send_recv_tensor_dict(self, send_tensor_dict, send_dst=None, recv_src=None, send_all_gather_group=None,
                              recv_all_gather_group=None):
        self.send_tensor_dict(send_tensor_dict)
        return self.recv_tensor_dict()

    # ---- object relay: external PP has one scheduler, nothing to relay -------------
    def send_object(self, obj, dst: int, async_send: bool = False, tag: int = 0):
        raise NotImplementedError("external PP: requests are not relayed between stages")

    def recv_object(self, src: int, tag: int = 0):
        raise NotImplementedError("external PP: requests are not relayed between stages")

    def barrier(self):
        return None

    def destroy(self) -> None:
        close = getattr(self.t, "close", None)
        if close is not None:
            close()


__all__ = ["ConnexPPGroup", "MSG_TYPE", "MISSING_HERE", "REPREFILLED"]

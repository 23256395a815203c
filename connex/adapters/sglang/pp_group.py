"""SGLang ``pp_group`` backed by the step protocol (external, elastic PP;
communication side only).

SGLang's scheduler reaches its pipeline neighbours only through
``scheduler.pp_group`` (a ``GroupCoordinator``): ``send_tensor_dict`` /
``recv_tensor_dict`` tagged ``"__msg_type__": "proxy"`` (hidden states going
forward) or ``"output"`` (sampled tokens coming back), plus the rank
properties.  :class:`ConnexPPGroup` serves that surface over a step transport
(:class:`connex.pp.endpoint.PipelineEndpoint`, or the in-process fakes of
:mod:`connex.pp.testing`) in the external topology, with one role object
per stage kind:

:class:`_Head` (stage 0, the only scheduler)
    a ``proxy`` send starts a step through :class:`connex.pp.link.Stage0Link`
    (correlation id, ``cx_ctx`` and finished ids attached); a receive returns
    the ``output`` of the oldest outstanding step -- SGLang consumes
    microbatch results in launch order.  Re-sends after a failover and the
    ``reprefill`` hook are Stage0Link's.

:class:`_Relay` (stages 1.., passive executors)
    a receive returns the next step's ``proxy`` dict after the KV ownership
    check: rows this stage holds no KV for are released and listed under
    :data:`MISSING_HERE` (the engine must not cache them).  The next send
    answers that step -- forwarded to the next stage, or from the last
    stage as the ``output`` back to stage 0 -- with the missing rows merged
    into ``cx_missing``.

The engine side (one scheduler on stage 0, stateless executors that load
only their layers, per-request KV accounting, re-prefill) is SGLang's.
Interface parity: ``connex/adapters/sglang/pp_group.py:65-195`` of the
reference (the GroupCoordinator surface and tags SGLang touches).
"""
from __future__ import annotations

import collections
import logging
from typing import Any, Callable, Optional, Sequence

from connex.pp.handover import CX_CTX, CX_MISSING, FINISHED, REQUEST_IDS, find_missing, merge_missing
from connex.pp.link import Stage0Link

MSG_TYPE = "__msg_type__"
MISSING_HERE = "__cx_missing_here__"     # stages 1..: rows this stage has no KV for
REPREFILLED = "__cx_reprefilled__"       # stage 0: rows the engine must recompute

_log = logging.getLogger("connex.adapters.sglang")


class _Done:
    """SGLang's P2P work handle (``.work.wait()``): a send here has been handed
    to the transport by the time it returns."""

    class _Work:
        def wait(self):
            return True

        def is_completed(self):
            return True

    def __init__(self):
        self.work = self._Work()


class _Head:
    def __init__(self, group: "ConnexPPGroup", recv_timeout_s, max_attempts):
        self.g = group
        self.link = Stage0Link(group.t, group.hooks, recv_timeout_s=recv_timeout_s, max_attempts=max_attempts,
                               log=group.log)
        self.launched: collections.deque = collections.deque()      # correlation ids, launch order

    def send(self, tensor_dict: dict) -> None:
        rids, computed = self.g.row_info() if self.g.row_info is not None else (None, None)
        self.launched.append(self.link.submit(dict(tensor_dict), rids, computed))

    def recv(self) -> dict:
        if not self.launched:
            raise RuntimeError("ConnexPPGroup: stage 0 receive without an outstanding step")
        reply = self.link.wait(self.launched.popleft())
        reply.setdefault(MSG_TYPE, "output")
        return reply

    def finished(self, request_ids: Sequence) -> None:
        self.link.finished(request_ids)


class _Relay:
    def __init__(self, group: "ConnexPPGroup"):
        self.g = group
        self.received: collections.deque = collections.deque()      # (reply context, step dict)

    def _ownership_check(self, td: dict) -> list:
        """Free finished requests; release and return the rows without KV here."""
        hooks = self.g.hooks
        if hooks is None:
            return []
        rids = td.get(REQUEST_IDS) or []
        scheduled = set(rids)
        ended = [r for r in td.get(FINISHED) or () if r not in scheduled]
        if ended:
            hooks.release(ended)
        lacking = find_missing(rids, td.get(CX_CTX), hooks.kv_held)
        if lacking:
            self.g.log.warning("stage %s: no KV here for %d of %d request(s)", self.g.t.stage_idx, len(lacking),
                               len(rids))
            hooks.release(lacking)
            self.g.stats["missing"] += len(lacking)
        return lacking

    def recv(self, timeout_s: Optional[float] = None) -> Optional[dict]:
        """The next step (waits for one; with ``timeout_s`` None when none came)."""
        td, ctx = None, None
        while td is None:
            td, ctx = self.g.t.recv_forward() if timeout_s is None else self.g.t.recv_forward(timeout_s)
            if td is None and timeout_s is not None:
                return None
        td[MISSING_HERE] = self._ownership_check(td)
        td.setdefault(MSG_TYPE, "proxy")
        self.received.append((ctx, td))
        return td

    def send(self, tensor_dict: dict) -> None:
        if not self.received:
            raise RuntimeError("ConnexPPGroup: a later stage sends only to answer a received step")
        ctx, step = self.received.popleft()
        out = {k: v for k, v in tensor_dict.items() if k != MISSING_HERE}
        union = merge_missing(step.get(CX_MISSING), step.get(MISSING_HERE))
        if union:
            out[CX_MISSING] = union
        if self.g.t.is_last:
            out[MSG_TYPE] = "output"
        else:
            for key in (REQUEST_IDS, CX_CTX, FINISHED):
                if key in step:
                    out.setdefault(key, step[key])
        self.g.t.send_reply(out, ctx)


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
        self.stats = {"sent": 0, "received": 0, "missing": 0}
        self._role = _Head(self, recv_timeout_s, max_attempts) if transport.is_first else _Relay(self)

    # ---------------------------------------------- GroupCoordinator surface
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
        if isinstance(self._role, _Head):
            self._role.finished(request_ids)

    def send_tensor_dict(self, tensor_dict: dict, dst: Optional[int] = None, all_gather_group: Any = None,
                         async_send: bool = False):
        """``all_gather_group`` is ignored: one sender per stage sends whole tensors."""
        self.stats["sent"] += 1
        self._role.send(tensor_dict)
        return [_Done()]

    def recv_tensor_dict(self, src: Optional[int] = None, all_gather_group: Any = None) -> dict:
        self.stats["received"] += 1
        return self._role.recv()

    def try_recv_tensor_dict(self, timeout_s: float) -> Optional[dict]:
        """Stages 1..: like ``recv_tensor_dict`` but gives up after ``timeout_s``
        (returns None) -- for a serving loop that must notice a stop request."""
        if isinstance(self._role, _Head):
            raise RuntimeError("stage 0 receives replies with recv_tensor_dict")
        td = self._role.recv(timeout_s)
        if td is not None:
            self.stats["received"] += 1
        return td

    def send_recv_tensor_dict(self, send_tensor_dict, send_dst=None, recv_src=None, send_all_gather_group=None,
                              recv_all_gather_group=None):
        self.send_tensor_dict(send_tensor_dict)
        return self.recv_tensor_dict()

    # ------------------------ object relay: external PP has a single scheduler
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

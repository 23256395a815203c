"""Engine-facing drivers of the pipeline step protocol (reference
``connex/pp/link.py:38-193``), usable on top of any :class:`StepTransport`.

* :class:`Stage0Link` -- submit a step (``cx_ctx`` / ``finished_req_ids``
  piggybacked), wait for its reply with per-step retries under the same
  correlation id, fast handover of other in-flight steps whose chain failed
  over, bounded attempts while the downstream is unhealthy, ``cx_missing``
  -> re-prefill / abort through :class:`EngineHooks`.
* :class:`StageWorker` -- receive, release finished requests, find rows
  whose KV this stage lacks, compute, send on with the merged ``cx_missing``.
"""
from __future__ import annotations

import logging
from typing import Callable, Optional, Sequence

from connex.pp.handover import (CX_CTX, CX_MISSING, FINISHED, REQUEST_IDS, FinishedOutbox, RewindBudget,
                                find_missing, merge_missing)
from connex.pp.steptrace import tr

_log = logging.getLogger("connex.pp.link")


class StepFailed(RuntimeError):
    """A step got no reply after all retries (no healthy downstream)."""


class Stage0Link:
    def __init__(self, transport, hooks=None, *, max_attempts: int = 5, recv_timeout_s: Optional[float] = None,
                 reprefill_max: int = 8, finished_repeat: int = 2, send_ctx: bool = True,
                 max_healthy_attempts: int = 1000, log: logging.Logger = _log):
        self.t = transport
        self.hooks = hooks
        self.max_attempts = max_attempts
        self.max_healthy_attempts = max_healthy_attempts
        self.recv_timeout_s = recv_timeout_s
        self.send_ctx = send_ctx
        self.rewinds = RewindBudget(reprefill_max)
        self.outbox = FinishedOutbox(finished_repeat)
        self.log = log
        self._sent: dict = {}
        self.stats = {"steps": 0, "retries": 0, "reprefilled": 0, "aborted": 0}

    @property
    def inflight(self) -> int:
        return getattr(self.t, "inflight", 1)

    def finished(self, request_ids: Sequence) -> None:
        self.outbox.add(request_ids)
        self.rewinds.forget(request_ids)

    def submit(self, tensor_dict: dict, request_ids: Optional[Sequence] = None,
               num_computed: Optional[Sequence[int]] = None) -> int:
        td = dict(tensor_dict)
        if request_ids is not None:
            td.setdefault(REQUEST_IDS, list(request_ids))
            if self.send_ctx and num_computed is not None:
                td[CX_CTX] = [int(n) for n in num_computed]
        fin = self.outbox.take()
        if fin:
            td[FINISHED] = fin
        corr = self.t.new_step_id()
        self._sent[corr] = td
        tr("s0_send", corr)
        self.t.send_step(td, corr)
        self.stats["steps"] += 1
        return corr

    def wait(self, corr: int) -> dict:
        attempts = 0
        while True:
            reply = self.t.recv_step(corr, self.recv_timeout_s)
            if reply is not None:
                break
            attempts += 1
            limit = self.max_healthy_attempts if self.t.downstream_healthy() else self.max_attempts
            if attempts >= limit:
                self.t.abandon_step(corr)
                self._sent.pop(corr, None)
                raise StepFailed(f"step {corr:x}: no reply after {attempts} attempts")
            self.stats["retries"] += 1
            tr("s0_resend", corr)
            self.t.send_step(self._sent[corr], corr)
            self._resend_stale(corr)
        tr("s0_reply", corr)
        self._sent.pop(corr, None)
        missing = reply.pop(CX_MISSING, None)
        if missing:
            again, abort = self.rewinds.split(missing)
            if self.hooks is not None:
                if again:
                    self.hooks.reprefill(again)
                if abort:
                    self.hooks.abort(abort)
            self.stats["reprefilled"] += len(again)
            self.stats["aborted"] += len(abort)
            reply["__cx_reprefilled__"] = again
            reply["__cx_aborted__"] = abort
        return reply

    def _resend_stale(self, current: int) -> None:
        """Other in-flight steps sent on a chain that failed over since are
        lost too: re-send them now, oldest first."""
        stale = getattr(self.t, "step_stale", None)
        if stale is None:
            return
        for c in sorted(c for c in self._sent if c != current):
            if stale(c):
                self.stats["retries"] += 1
                self.t.send_step(self._sent[c], c)

    def step(self, tensor_dict: dict, request_ids=None, num_computed=None) -> dict:
        return self.wait(self.submit(tensor_dict, request_ids, num_computed))


class StageWorker:
    """``compute(td, missing) -> dict`` is the stage's forward; rows of
    ``missing`` requests were released and must not be cached."""

    def __init__(self, transport, hooks, compute: Callable[[dict, list], dict], *,
                 commit: Optional[Callable[[dict, list], None]] = None, log: logging.Logger = _log):
        self.t = transport
        self.hooks = hooks
        self.compute = compute
        self.commit = commit
        self.log = log
        self.stats = {"steps": 0, "missing": 0, "released_finished": 0}

    def serve_one(self) -> bool:
        td, ctx = self.t.recv_forward()
        if td is None:
            return False
        self.serve(td, ctx)
        return True

    def serve(self, td: dict, ctx) -> None:
        """Process one received step (``recv_forward`` output) and send it on."""
        seq = ctx[0] if isinstance(ctx, tuple) and ctx else 0
        tr(f"s{getattr(self.t, 'stage_idx', 'x')}_recv", seq)
        self.stats["steps"] += 1
        rids = td.get(REQUEST_IDS) or []
        fin = td.get(FINISHED)
        if fin:
            live = set(rids)
            done = [r for r in fin if r not in live]  # scheduled in this very step: not yet
            if done:
                self.hooks.release(done)
                self.stats["released_finished"] += len(done)
        mine = find_missing(rids, td.get(CX_CTX), self.hooks.kv_held)
        if mine:
            self.log.warning("stage %s: %d/%d requests have no KV here", getattr(self.t, "stage_idx", "?"),
                             len(mine), len(rids))
            self.hooks.release(mine)
            self.stats["missing"] += len(mine)
        out = dict(self.compute(td, mine) or {})
        if self.commit is not None:
            self.commit(td, mine)
        merged = merge_missing(td.get(CX_MISSING), mine)
        if merged:
            out[CX_MISSING] = merged
        if not self.t.is_last:
            for k in (REQUEST_IDS, CX_CTX, FINISHED):
                if k in td and k not in out:
                    out[k] = td[k]
        tr(f"s{getattr(self.t, 'stage_idx', 'x')}_send", seq)
        self.t.send_reply(out, ctx)

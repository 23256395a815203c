"""Engine-facing drivers of the pipeline step protocol, on top of any
:class:`connex.pp.hooks.StepTransport`.

:class:`Stage0Link` (the first stage)
    ``submit`` stamps a step with the per-row context lengths (``cx_ctx``)
    and the finished ids to piggyback, sends it and returns its correlation
    id; ``wait`` collects the reply.  A reply that does not arrive within the
    receive timeout is re-sent under the same id -- as many times as the
    retry policy allows (many while the downstream looks healthy, few when it
    does not) -- and any other in-flight step whose chain has failed over
    since it was sent is re-sent at the same moment (fast handover).
    Requests reported in ``cx_missing`` are re-prefilled through the engine
    hooks, or aborted once their re-prefill budget is used up.

:class:`StageWorker` (every later stage)
    receives a step, frees the KV of requests finished upstream, detects the
    rows whose KV this replica lacks (releases them and computes the batch
    without caching those rows), and sends the result on with the union of
    the missing ids.

Behavioural parity: ``connex/pp/link.py:38-193`` of the reference.
"""
from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

from connex.pp.handover import (CX_CTX, CX_MISSING, FINISHED, REQUEST_IDS, FinishedOutbox, RewindBudget,
                                find_missing, merge_missing)
from connex.pp.steptrace import tr

_log = logging.getLogger("connex.pp.link")

# keys of the original step that a middle stage forwards with its output
_FORWARDED = (REQUEST_IDS, CX_CTX, FINISHED)


class StepFailed(RuntimeError):
    """A step got no reply after every allowed retry (no healthy downstream)."""


@dataclass
class _Pending:
    """A step stage 0 sent and has not yet received the reply of."""

    payload: dict
    sent_at: float = field(default_factory=time.monotonic)
    resends: int = 0
    first_sent: float = field(default_factory=time.monotonic)

    @property
    def size(self) -> int:
        """Scheduled tokens (``n_new``) or rows of the step, for comparing step times."""
        n_new = self.payload.get("n_new")
        if isinstance(n_new, (list, tuple)):
            return int(sum(int(x) for x in n_new))
        return len(self.payload.get(REQUEST_IDS) or ())


class Stage0Link:
    def __init__(self, transport, hooks=None, *, max_attempts: int = 5, recv_timeout_s: Optional[float] = None,
                 reprefill_max: int = 8, finished_repeat: int = 2, send_ctx: bool = True,
                 max_healthy_attempts: int = 1000, log: logging.Logger = _log):
        self.t = transport
        self.hooks = hooks
        self.max_attempts = max_attempts                  # retries while the downstream looks dead
        self.max_healthy_attempts = max_healthy_attempts  # ... and while it looks healthy (slow step)
        self.recv_timeout_s = recv_timeout_s
        self.send_ctx = send_ctx
        self.rewinds = RewindBudget(reprefill_max)
        self.outbox = FinishedOutbox(finished_repeat)
        self.log = log
        self._pending: Dict[int, _Pending] = {}
        self.step_listeners: List[Callable[[float, int], None]] = []    # (seconds, size) per completed step
        self.stats = {"steps": 0, "retries": 0, "reprefilled": 0, "aborted": 0}

    @property
    def inflight(self) -> int:
        return getattr(self.t, "inflight", 1)

    def outstanding(self) -> List[int]:
        """Correlation ids of the steps awaiting a reply, oldest first."""
        return sorted(self._pending)

    def pending_steps(self) -> List[tuple]:
        """(corr, first sent at, size) of every step awaiting its reply."""
        return [(c, p.first_sent, p.size) for c, p in list(self._pending.items())]

    def finished(self, request_ids: Sequence) -> None:
        """Requests stage 0 finished: tell the downstream stages, forget their budget."""
        self.outbox.add(request_ids)
        self.rewinds.forget(request_ids)

    def _stamp(self, tensor_dict: dict, request_ids, num_computed) -> dict:
        step = dict(tensor_dict)
        if request_ids is not None:
            step.setdefault(REQUEST_IDS, list(request_ids))
            if self.send_ctx and num_computed is not None:
                step[CX_CTX] = [int(n) for n in num_computed]
        done = self.outbox.take()
        if done:
            step[FINISHED] = done
        return step

    def submit(self, tensor_dict: dict, request_ids: Optional[Sequence] = None,
               num_computed: Optional[Sequence[int]] = None) -> int:
        step = self._stamp(tensor_dict, request_ids, num_computed)
        corr = self.t.new_step_id()
        self._pending[corr] = _Pending(step)
        tr("s0_send", corr)
        self.t.send_step(step, corr)
        self.stats["steps"] += 1
        return corr

    def _resend(self, corr: int) -> None:
        p = self._pending[corr]
        p.resends += 1
        p.sent_at = time.monotonic()
        self.stats["retries"] += 1
        self.t.send_step(p.payload, corr)

    def _retry_budget(self) -> int:
        return self.max_healthy_attempts if self.t.downstream_healthy() else self.max_attempts

    def _hand_over_others(self, waiting_on: int) -> None:
        """Steps sent on a chain that has failed over since are lost too:
        re-send them now, oldest first, rather than waiting for their own
        timeouts."""
        is_stale = getattr(self.t, "step_stale", None)
        if is_stale is None:
            return
        for corr in self.outstanding():
            if corr != waiting_on and is_stale(corr):
                self._resend(corr)

    def _settle_missing(self, reply: dict) -> None:
        missing = reply.pop(CX_MISSING, None)
        if not missing:
            return
        again, give_up = self.rewinds.split(missing)
        if self.hooks is not None:
            if again:
                self.hooks.reprefill(again)
            if give_up:
                self.hooks.abort(give_up)
        self.stats["reprefilled"] += len(again)
        self.stats["aborted"] += len(give_up)
        reply["__cx_reprefilled__"] = again
        reply["__cx_aborted__"] = give_up

    def wait(self, corr: int) -> dict:
        timeouts = 0
        reply = self.t.recv_step(corr, self.recv_timeout_s)
        while reply is None:
            timeouts += 1
            if timeouts >= self._retry_budget():
                self.t.abandon_step(corr)
                self._pending.pop(corr, None)
                raise StepFailed(f"step {corr:x}: no reply after {timeouts} attempts")
            tr("s0_resend", corr)
            self._resend(corr)
            self._hand_over_others(corr)
            reply = self.t.recv_step(corr, self.recv_timeout_s)
        tr("s0_reply", corr)
        done = self._pending.pop(corr, None)
        if done is not None:
            for listener in list(self.step_listeners):
                listener(time.monotonic() - done.first_sent, done.size)
        self._settle_missing(reply)
        return reply

    def step(self, tensor_dict: dict, request_ids=None, num_computed=None) -> dict:
        return self.wait(self.submit(tensor_dict, request_ids, num_computed))


class StageWorker:
    """A downstream stage's loop body.  ``compute(td, missing) -> dict`` is
    the stage's forward; rows of the ``missing`` requests were released and
    must not be cached.  ``commit(td, missing)`` (optional) records what the
    stage now holds (e.g. :meth:`connex.pp.handover.KVLedger.commit`)."""

    def __init__(self, transport, hooks, compute: Callable[[dict, list], dict], *,
                 commit: Optional[Callable[[dict, list], None]] = None, log: logging.Logger = _log):
        self.t = transport
        self.hooks = hooks
        self.compute = compute
        self.commit = commit
        self.log = log
        self.stats = {"steps": 0, "missing": 0, "released_finished": 0}

    @property
    def _tag(self) -> str:
        return f"s{getattr(self.t, 'stage_idx', 'x')}"

    def serve_one(self) -> bool:
        """Serve one step; False when the transport returned nothing."""
        td, ctx = self.t.recv_forward()
        if td is None:
            return False
        self.serve(td, ctx)
        return True

    def _free_finished(self, td: dict, scheduled: List) -> None:
        # a finished id that is also scheduled in this very step is still in use
        done = [r for r in (td.get(FINISHED) or ()) if r not in set(scheduled)]
        if done:
            self.hooks.release(done)
            self.stats["released_finished"] += len(done)

    def _lacking(self, td: dict, scheduled: List) -> List:
        lacking = find_missing(scheduled, td.get(CX_CTX), self.hooks.kv_held)
        if lacking:
            self.log.warning("stage %s: %d/%d requests have no KV here", getattr(self.t, "stage_idx", "?"),
                             len(lacking), len(scheduled))
            self.hooks.release(lacking)
            self.stats["missing"] += len(lacking)
        return lacking

    def serve(self, td: dict, ctx) -> None:
        """Process one received step (a ``recv_forward`` result) and send it on."""
        seq = ctx[0] if isinstance(ctx, tuple) and ctx else 0
        tr(self._tag + "_recv", seq)
        self.stats["steps"] += 1
        scheduled = list(td.get(REQUEST_IDS) or [])
        self._free_finished(td, scheduled)
        lacking = self._lacking(td, scheduled)
        out = dict(self.compute(td, lacking) or {})
        if self.commit is not None:
            self.commit(td, lacking)
        union = merge_missing(td.get(CX_MISSING), lacking)
        if union:
            out[CX_MISSING] = union
        if not self.t.is_last:
            out.update({k: td[k] for k in _FORWARDED if k in td and k not in out})
        tr(self._tag + "_send", seq)
        self.t.send_reply(out, ctx)

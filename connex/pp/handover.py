"""In-flight handover rules of the pipeline step protocol (pure Python).

When a replica of a downstream stage dies, stage 0 re-sends the in-flight
steps to another replica, which may not hold the KV of every request in the
batch.  Stage 0 piggybacks each row's context length (``cx_ctx``); a stage
that holds less than that (``find_missing``) releases those requests, still
runs the batch (shapes are fixed) without caching their rows, and reports
their ids in ``cx_missing``; the last stage returns the union to stage 0,
which discards the tokens sampled for them and re-prefills prompt +
generated tokens on the current chain, aborting a request after
``max_rewinds`` re-prefills.  Finished ids travel downstream as
``finished_req_ids`` on ``repeat`` consecutive steps.
Reference: ``connex/pp/handover.py:34-149``.
"""
from __future__ import annotations

from collections import deque
from typing import Callable, Iterable, List, Optional, Sequence, Tuple

CX_CTX = "cx_ctx"
CX_MISSING = "cx_missing"
FINISHED = "finished_req_ids"
REQUEST_IDS = "request_ids"


def find_missing(request_ids: Sequence, ctx: Optional[Sequence[int]], held: Callable[[object], int]) -> list:
    """Requests whose context stage 0 reports (ctx > 0) but this stage lacks."""
    if not request_ids or ctx is None:
        return []
    out = []
    for i, rid in enumerate(request_ids):
        c = int(ctx[i]) if i < len(ctx) else 0
        if c > 0 and held(rid) < c:
            out.append(rid)
    return out


def merge_missing(upstream: Optional[Sequence], mine: Optional[Sequence]) -> Optional[list]:
    """Order-preserving union of upstream and local missing ids."""
    if not upstream:
        return list(mine) if mine else None
    if not mine:
        return list(upstream)
    out = list(upstream)
    seen = set(out)
    out += [r for r in mine if r not in seen]
    return out


def blank_rows(rows: Sequence, request_ids: Sequence, missing: Iterable) -> list:
    miss = set(missing)
    return [[] if i < len(request_ids) and request_ids[i] in miss else row for i, row in enumerate(rows)]


class KVLedger:
    """Tokens of each request this stage computed itself (never shrinks)."""

    def __init__(self, is_live: Optional[Callable[[object], bool]] = None):
        self.kv_len: dict = {}
        self.is_live = is_live

    def kv_held(self, rid) -> int:
        if self.is_live is not None and not self.is_live(rid):
            return 0
        return self.kv_len.get(rid, 0)

    def commit(self, request_ids: Sequence, ctx: Optional[Sequence[int]],
               num_scheduled: Optional[Sequence[int]] = None, missing: Iterable = ()) -> None:
        if not request_ids or ctx is None:
            return
        miss = set(missing or ())
        for i, rid in enumerate(request_ids):
            if rid in miss:
                continue
            c = int(ctx[i]) if i < len(ctx) else 0
            n = int(num_scheduled[i]) if num_scheduled is not None and i < len(num_scheduled) else 1
            if c == 0 or c + n > self.kv_len.get(rid, 0):
                self.kv_len[rid] = c + n

    def forget(self, rids: Iterable) -> None:
        for r in rids:
            self.kv_len.pop(r, None)


class FinishedOutbox:
    """Stage 0: finished ids piggybacked on the next ``repeat`` sends."""

    def __init__(self, repeat: int = 2):
        self.repeat = max(1, int(repeat))
        self._q: deque = deque()

    def add(self, rids: Iterable) -> None:
        self._q.extend([r, self.repeat] for r in rids)

    def take(self) -> Optional[list]:
        if not self._q:
            return None
        out = [e[0] for e in self._q]
        for e in self._q:
            e[1] -= 1
        self._q = deque(e for e in self._q if e[1] > 0)
        return out


class RewindBudget:
    """Stage 0: re-prefill count per request; past ``max_rewinds`` -> abort."""

    def __init__(self, max_rewinds: int = 8):
        self.max_rewinds = max_rewinds
        self.count: dict = {}

    def split(self, missing: Iterable) -> Tuple[List, List]:
        again, abort = [], []
        for rid in missing:
            n = self.count.get(rid, 0) + 1
            self.count[rid] = n
            (abort if n > self.max_rewinds else again).append(rid)
        return again, abort

    def forget(self, rids: Iterable) -> None:
        for r in rids:
            self.count.pop(r, None)

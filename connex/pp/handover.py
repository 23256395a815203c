"""In-flight handover rules of the pipeline step protocol (pure Python).

When a downstream replica dies, stage 0 re-sends its in-flight steps to
another replica, which may not hold the KV of every request in the batch.
The protocol repairs this without moving KV:

* with every step stage 0 sends ``cx_ctx``: for each row, the number of
  tokens of that request computed before this step;
* a stage that holds fewer tokens than that for a request (``find_missing``)
  releases the request, still runs the batch (its shape is fixed) but does
  not cache those rows, and adds their ids to ``cx_missing``;
* the last stage returns the union of ``cx_missing`` to stage 0, which
  throws away the tokens sampled for those rows and re-prefills prompt plus
  generated tokens on the current chain -- at most ``max_rewinds`` times per
  request before aborting it (``RewindBudget``);
* ids of finished requests ride downstream as ``finished_req_ids`` on
  ``repeat`` consecutive steps (``FinishedOutbox``) so the other stages
  free their KV early.

Keys and semantics follow ``connex/pp/handover.py:34-149`` of the
reference, so stages built on either implementation interoperate.
"""
from __future__ import annotations

from collections import Counter
from typing import Callable, Dict, Iterable, Iterator, List, Optional, Sequence, Tuple

CX_CTX = "cx_ctx"
CX_MISSING = "cx_missing"
FINISHED = "finished_req_ids"
REQUEST_IDS = "request_ids"


def _with_ctx(request_ids: Sequence, ctx: Sequence[int]) -> Iterator[Tuple[object, int]]:
    """(request id, context length) per row; rows past the end of ``ctx`` count as 0."""
    n = len(ctx)
    for i, rid in enumerate(request_ids):
        yield rid, (int(ctx[i]) if i < n else 0)


def find_missing(request_ids: Sequence, ctx: Optional[Sequence[int]], held: Callable[[object], int]) -> list:
    """Requests that stage 0 says have context (ctx > 0) but of which this
    stage holds fewer tokens.  Without ``ctx`` nothing can be checked."""
    if ctx is None or not request_ids:
        return []
    return [rid for rid, c in _with_ctx(request_ids, ctx) if c > 0 and held(rid) < c]


def merge_missing(upstream: Optional[Sequence], mine: Optional[Sequence]) -> Optional[list]:
    """Union of the earlier stages' missing ids and this stage's, first
    occurrence order kept; None when both are empty."""
    merged = list(dict.fromkeys([*(upstream or ()), *(mine or ())]))
    return merged or None


def blank_rows(rows: Sequence, request_ids: Sequence, missing: Iterable) -> list:
    """``rows`` with the entries of missing requests replaced by empty lists."""
    gone = set(missing)
    ids = list(request_ids)
    return [[] if i < len(ids) and ids[i] in gone else row for i, row in enumerate(rows)]


class KVLedger:
    """How many tokens of each request this stage has computed and cached.

    An entry only grows (a re-executed older step cannot shrink it), except
    that a step starting at context 0 -- a fresh prefill -- resets it.
    ``is_live(rid)`` (optional) lets the engine veto entries whose KV it has
    since dropped."""

    def __init__(self, is_live: Optional[Callable[[object], bool]] = None):
        self.kv_len: Dict[object, int] = {}
        self.is_live = is_live

    def kv_held(self, rid) -> int:
        if self.is_live is not None and not self.is_live(rid):
            return 0
        return self.kv_len.get(rid, 0)

    def commit(self, request_ids: Sequence, ctx: Optional[Sequence[int]],
               num_scheduled: Optional[Sequence[int]] = None, missing: Iterable = ()) -> None:
        """Record a computed step: row i now covers ``ctx[i] + num_scheduled[i]``
        tokens (1 per row when ``num_scheduled`` is absent); rows of missing
        requests were not cached and are skipped."""
        if ctx is None or not request_ids:
            return
        skip = set(missing or ())
        steps = list(num_scheduled) if num_scheduled is not None else []
        for i, (rid, c) in enumerate(_with_ctx(request_ids, ctx)):
            if rid in skip:
                continue
            covered = c + (int(steps[i]) if i < len(steps) else 1)
            if c == 0:
                self.kv_len[rid] = covered
            else:
                self.kv_len[rid] = max(covered, self.kv_len.get(rid, 0))

    def forget(self, rids: Iterable) -> None:
        for rid in rids:
            self.kv_len.pop(rid, None)


class FinishedOutbox:
    """Stage 0's finished ids, each attached to the next ``repeat`` sends
    (so one lost step does not leave a downstream stage holding KV)."""

    def __init__(self, repeat: int = 2):
        self.repeat = max(1, int(repeat))
        self._left: Dict[object, int] = {}      # id -> sends still to carry it

    def add(self, rids: Iterable) -> None:
        for rid in rids:
            self._left[rid] = self.repeat

    def take(self) -> Optional[list]:
        if not self._left:
            return None
        out = list(self._left)
        self._left = {rid: n - 1 for rid, n in self._left.items() if n > 1}
        return out


class RewindBudget:
    """Stage 0's re-prefill count per request: ``split`` returns the requests
    that may be re-prefilled once more and those that used up
    ``max_rewinds`` and must be aborted."""

    def __init__(self, max_rewinds: int = 8):
        self.max_rewinds = max_rewinds
        self.count: Counter = Counter()

    def split(self, missing: Iterable) -> Tuple[List, List]:
        retry: List = []
        give_up: List = []
        for rid in missing:
            self.count[rid] += 1
            (retry if self.count[rid] <= self.max_rewinds else give_up).append(rid)
        return retry, give_up

    def forget(self, rids: Iterable) -> None:
        for rid in rids:
            self.count.pop(rid, None)

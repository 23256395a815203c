"""Step-protocol bookkeeping that never touches a transport.

A pipeline step carries a correlation id ``corr = incarnation << 32 | seq``
chosen by stage 0 (a random 32-bit incarnation per stage-0 process and a
running sequence number).  A re-sent step keeps its id and later stages echo
it, which gives three properties:

* replies can be matched to steps while K steps are in flight;
* a retried step is answered from the stage's reply cache, not recomputed;
* a step that is K or more sequence numbers behind the newest one seen from
  the same incarnation is stale and dropped.

Behavioural parity: ``connex/pp/steps.py:21-91`` of the reference (same
class names and semantics; the data structures here are this module's own).
"""
from __future__ import annotations

import os
from typing import Any, Callable, Dict, Optional

_SEQ_MASK = (1 << 32) - 1


def _split(corr: int):
    return corr >> 32, corr & _SEQ_MASK


class CorrFilter:
    """Admission test for incoming step ids.

    For each stage-0 incarnation the filter remembers the newest sequence
    number seen.  ``window`` is how many steps that sender keeps in flight:
    ids inside the window may arrive out of order (a per-step retry routed
    around a failed replica), ids ``window`` or more behind the newest are
    stale.  At most ``cap`` incarnations are remembered; the one heard from
    least recently is forgotten first (dict order is kept as recency)."""

    def __init__(self, cap: int = 64, window: int = 1):
        self.cap = int(cap)
        self.window = max(1, int(window))
        self._newest: Dict[int, int] = {}

    def accept(self, corr: Optional[int]) -> bool:
        if not corr:
            return True                      # a sender without ids: nothing to judge
        inc, seq = _split(corr)
        newest = self._newest.pop(inc, None)  # re-inserted below, as the most recent
        stale = newest is not None and newest - seq >= self.window
        self._newest[inc] = seq if newest is None else max(newest, seq)
        if len(self._newest) > self.cap:
            del self._newest[next(iter(self._newest))]
        return not stale


class StepIds:
    """Correlation ids of one stage-0 process: ``base + 1``, ``base + 2``, ...
    where ``base`` holds a random 32-bit incarnation in its high half."""

    def __init__(self, base: Optional[int] = None):
        if base is None:
            base = int.from_bytes(os.urandom(4), "big") << 32
        self.base = base
        self.seq = 0

    def next(self) -> int:
        self.seq += 1
        return self.base + self.seq


class ReplyCache:
    """The newest ``k`` replies of a stage, keyed by correlation id, so a
    duplicate step is answered again instead of recomputed.

    ``on_evict(entry)`` is called for every entry that leaves the cache,
    whether pushed out by newer replies or replaced under the same id (the
    PP endpoint unpins the entry's send-ring region there)."""

    def __init__(self, k: int = 1, on_evict: Optional[Callable[[Any], None]] = None):
        self.k = max(1, int(k))
        self.on_evict = on_evict
        self.entries: Dict[int, Any] = {}    # insertion order = age

    def _drop(self, entry) -> None:
        if self.on_evict is not None:
            self.on_evict(entry)

    def put(self, corr: int, entry: Any) -> None:
        if corr in self.entries:
            self._drop(self.entries.pop(corr))
        self.entries[corr] = entry
        overflow = len(self.entries) - self.k
        if overflow > 0:
            for old in list(self.entries)[:overflow]:
                self._drop(self.entries.pop(old))

    def get(self, corr):
        return self.entries.get(corr)

    def __contains__(self, corr) -> bool:
        return corr in self.entries

    def __len__(self) -> int:
        return len(self.entries)

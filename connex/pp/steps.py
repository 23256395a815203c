"""Step-protocol bookkeeping that never touches a transport.

Stage 0 stamps every pipeline step with ``corr = incarnation << 32 | seq``
and re-sends a step under the same id; later stages echo it.  That yields
reply matching with K steps in flight, idempotent retries (a duplicate is
answered from :class:`ReplyCache`), and stale suppression
(:class:`CorrFilter`: an id K or more behind the newest id of the same
incarnation is dropped).  Reference: ``connex/pp/steps.py:21-91``.
"""
from __future__ import annotations

import os
from collections import OrderedDict
from typing import Any, Callable, Optional


class CorrFilter:
    """Newest seq seen per stage-0 incarnation; ``accept`` drops ids that are
    ``window`` or more behind it (``window`` = steps the sender keeps in flight)."""

    def __init__(self, cap: int = 64, window: int = 1):
        self.cap = cap
        self.window = max(1, int(window))
        self.hi: "OrderedDict[int, int]" = OrderedDict()

    def accept(self, corr: Optional[int]) -> bool:
        if not corr:
            return True
        inc, seq = corr >> 32, corr & 0xFFFFFFFF
        newest = self.hi.get(inc)
        if newest is not None and seq + self.window <= newest:
            return False
        self.hi[inc] = seq if newest is None else max(newest, seq)
        self.hi.move_to_end(inc)
        while len(self.hi) > self.cap:
            self.hi.popitem(last=False)
        return True


class StepIds:
    """Correlation-id allocator of a stage-0 process (random 32-bit incarnation)."""

    def __init__(self, base: Optional[int] = None):
        self.base = (int.from_bytes(os.urandom(4), "big") << 32) if base is None else base
        self.seq = 0

    def next(self) -> int:
        self.seq += 1
        return self.base + self.seq


class ReplyCache:
    """Last ``k`` replies by correlation id; ``on_evict`` runs for every
    evicted or replaced entry (e.g. to unpin its send-ring region)."""

    def __init__(self, k: int = 1, on_evict: Optional[Callable[[Any], None]] = None):
        self.k = max(1, int(k))
        self.on_evict = on_evict
        self.entries: "OrderedDict[int, Any]" = OrderedDict()

    def put(self, corr: int, entry: Any) -> None:
        old = self.entries.pop(corr, None)
        if old is not None and self.on_evict:
            self.on_evict(old)
        self.entries[corr] = entry
        while len(self.entries) > self.k:
            _, e = self.entries.popitem(last=False)
            if self.on_evict:
                self.on_evict(e)

    def get(self, corr):
        return self.entries.get(corr)

    def __contains__(self, corr) -> bool:
        return corr in self.entries

    def __len__(self) -> int:
        return len(self.entries)

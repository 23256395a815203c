"""Send-ring bookkeeping of the PP data plane (pure Python).

An outgoing step is staged in a region of a registered send ring; the
receiver one-sided-reads it and acks the region's token (``CXACK``).  A
region is reused only once acked, or after a safety deadline when the
receiver died without acking; regions of replies that may be re-sent for a
duplicate request stay pinned while they sit in the reply cache.  When the
ring has no free span, the sender falls back to a temporary buffer that is
tracked the same way.  Reference: ``connex/pp/ring.py:16-106``.
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple


class Lease:
    __slots__ = ("start", "end", "deadline", "acked", "pinned", "obj", "want_ack")

    def __init__(self, start: int, end: int, deadline: float, want_ack: bool, obj=None):
        self.start, self.end, self.deadline = start, end, deadline
        self.acked = False
        self.pinned = False
        self.obj = obj
        self.want_ack = want_ack


class RegionTable:
    def __init__(self, size: int, token_base: Optional[int] = None):
        self.size = size
        self.head = 0
        self.leases: dict = {}
        self._seq = 0
        self.base = (int.from_bytes(os.urandom(4), "big") << 32) if token_base is None else token_base
        self.expired_unacked = 0

    def _token(self) -> int:
        self._seq = ((self._seq + 1) & 0xFFFFFFFF) or 1
        return self.base | self._seq

    @staticmethod
    def _busy(lease: Lease, now: float) -> bool:
        return lease.pinned or (not lease.acked and lease.deadline > now)

    def alloc(self, n: int, now: float, hold_s: float, want_ack: bool) -> Optional[Tuple[int, int]]:
        """(offset, token) of a free ring span of ``n`` bytes, or None."""
        if n > self.size:
            return None
        start = self.head if self.head + n <= self.size else 0
        end = start + n
        for l in self.leases.values():
            if l.obj is None and self._busy(l, now) and start < l.end and l.start < end:
                return None
        tok = self._token()
        self.leases[tok] = Lease(start, end, now + hold_s, want_ack)
        self.head = end
        return start, tok

    def add_temp(self, obj, now: float, hold_s: float, want_ack: bool) -> int:
        tok = self._token()
        self.leases[tok] = Lease(0, 0, now + hold_s, want_ack, obj)
        return tok

    def ack(self, tok: int) -> bool:
        l = self.leases.get(tok)
        if l is None:
            return False
        l.acked = True
        return True

    def pin(self, tok: int) -> None:
        l = self.leases.get(tok)
        if l is not None:
            l.pinned = True

    def unpin(self, tok: int) -> None:
        l = self.leases.get(tok)
        if l is not None:
            l.pinned = False

    def awaiting_ack(self) -> bool:
        return any(l.want_ack and not l.acked for l in self.leases.values())

    def collect(self, now: float) -> List:
        """Forget free leases; returns temp buffers that may now be released."""
        freed = []
        for tok, l in list(self.leases.items()):
            if self._busy(l, now):
                continue
            if l.want_ack and not l.acked:
                self.expired_unacked += 1
            del self.leases[tok]
            if l.obj is not None:
                freed.append(l.obj)
        return freed

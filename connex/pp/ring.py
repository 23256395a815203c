"""Send-ring bookkeeping of the PP data plane (pure Python).

A step's tensors are staged in a span of a registered send ring; the
receiver one-sided-reads the span and acknowledges its token (``CXACK``).
The sender may write over a span again only when it is *free*:

* it was acknowledged and is not pinned, or
* its safety deadline passed (the receiver died without acknowledging);
* a pinned span (a reply that may be re-sent for a duplicate step) is never
  free until unpinned.

When no free span fits, the caller stages into a temporary buffer instead;
the table tracks that buffer under a token too and hands it back from
:meth:`RegionTable.collect` once it is free.

The ring is filled in allocation order: a cursor advances through the ring
and wraps to offset 0 when the next span would not fit before the end.
Behavioural parity: ``connex/pp/ring.py:16-106`` of the reference (names and
rules kept; the structures here are this module's own).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple


@dataclass
class Lease:
    """One staged send: a ring span ``[start, end)`` or a temporary buffer (``obj``)."""

    start: int
    end: int
    deadline: float
    want_ack: bool
    obj: Any = None
    acked: bool = False
    pinned: bool = False

    def held(self, now: float) -> bool:
        """True while the span must not be reused."""
        if self.pinned:
            return True
        return not self.acked and now < self.deadline

    def overlaps(self, lo: int, hi: int) -> bool:
        return self.obj is None and lo < self.end and self.start < hi


class RegionTable:
    """Spans of one send ring of ``size`` bytes, keyed by 64-bit tokens
    ``token_base | n`` (n a 32-bit counter that skips 0)."""

    def __init__(self, size: int, token_base: Optional[int] = None):
        self.size = int(size)
        self.base = (int.from_bytes(os.urandom(4), "big") << 32) if token_base is None else token_base
        self.head = 0                       # where the next span starts (before wrapping)
        self.leases: Dict[int, Lease] = {}
        self.expired_unacked = 0            # spans reclaimed by deadline, never acknowledged
        self._counter = 0

    def _new_token(self) -> int:
        self._counter = self._counter % 0xFFFFFFFF + 1
        return self.base | self._counter

    def _register(self, lease: Lease) -> int:
        tok = self._new_token()
        self.leases[tok] = lease
        return tok

    def alloc(self, n: int, now: float, hold_s: float, want_ack: bool) -> Optional[Tuple[int, int]]:
        """Reserve ``n`` bytes; returns ``(offset, token)`` or None when the
        span at the cursor (after wrapping if needed) is still held."""
        if n > self.size:
            return None
        lo = 0 if self.head + n > self.size else self.head
        hi = lo + n
        if any(l.overlaps(lo, hi) and l.held(now) for l in self.leases.values()):
            return None
        self.head = hi
        return lo, self._register(Lease(lo, hi, now + hold_s, want_ack))

    def add_temp(self, obj, now: float, hold_s: float, want_ack: bool) -> int:
        """Track a temporary buffer staged outside the ring; returns its token."""
        return self._register(Lease(0, 0, now + hold_s, want_ack, obj=obj))

    def ack(self, tok: int) -> bool:
        lease = self.leases.get(tok)
        if lease is not None:
            lease.acked = True
        return lease is not None

    def pin(self, tok: int) -> None:
        self._set_pin(tok, True)

    def unpin(self, tok: int) -> None:
        self._set_pin(tok, False)

    def _set_pin(self, tok: int, value: bool) -> None:
        lease = self.leases.get(tok)
        if lease is not None:
            lease.pinned = value

    def awaiting_ack(self) -> bool:
        return any(l.want_ack and not l.acked for l in self.leases.values())

    def collect(self, now: float) -> List:
        """Drop every free lease; returns the temporary buffers among them
        (the caller may release those now)."""
        free = [tok for tok, l in self.leases.items() if not l.held(now)]
        buffers = []
        for tok in free:
            lease = self.leases.pop(tok)
            self.expired_unacked += lease.want_ack and not lease.acked
            if lease.obj is not None:
                buffers.append(lease.obj)
        return buffers

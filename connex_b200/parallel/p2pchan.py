"""GPU-driven point-to-point channels over NVLink peer memory (no NCCL).

A channel from endpoint A to endpoint B is a ring of ``slots`` x
``slot_bytes`` in B's GPU memory plus two u32 counters: ``ready`` (in B's
memory; A's copy kernel adds its CTA count when a ring message has landed)
and ``credit`` (in A's memory; B stores the sequence number of the last
message it has copied out).  Everything is stream-ordered on both sides:

* sender, message ``k``: one kernel waits (bounded) until
  ``credit >= k - slots``, stores the tensors straight into B's ring slot
  over the peer mapping and releases ``ready`` (+1 per CTA, system scope);
* receiver: one kernel waits (bounded) until ``ready`` reaches the running
  target, copies the slot out into the destination tensors, and its last
  CTA stores ``credit = k`` into A's memory (``chan.cu``).

Messages larger than a slot go as consecutive slot-sized pieces.  Both sides
derive the pieces and CTA counts from the tensor sizes, so only the tensor
layout has to travel on the control channel (the step protocol's signal).
Handles are exchanged through a ``torch.distributed`` store under
``cxch/<sender>><receiver>/``.  ``ChanLinks`` has the interface of
:class:`connex_b200.parallel.pplink.PairLinks` (``open_tx`` / ``open_rx``
returning links with ``send`` / ``recv`` / ``done_event``), so a pipeline
endpoint uses either data plane unchanged.
"""
from __future__ import annotations

import pickle
import threading
from datetime import timedelta
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from connex_b200 import ops
from connex_b200.parallel.peer import PeerHandle, PeerMapper, export_tensor, shared_empty

ALIGN = 256
CHAN_CTAS = 64


def _layout(tensors: Sequence[torch.Tensor]) -> Tuple[List[Tuple[int, int]], int]:
    offs, total = [], 0
    for t in tensors:
        n = t.numel() * t.element_size()
        if n % 16:
            raise ValueError("channel tensors must be a multiple of 16 bytes")
        offs.append((total, n))
        total += -(-n // ALIGN) * ALIGN
    return offs, total


def _pieces(offs, total: int, slot_bytes: int):
    """[(piece start, piece len, [(tensor idx, t_off, p_off, n)])] covering the layout."""
    out = []
    for p0 in range(0, max(total, 1), slot_bytes):
        p1 = min(total, p0 + slot_bytes)
        parts = []
        for i, (o, n) in enumerate(offs):
            a, b = max(o, p0), min(o + n, p1)
            if a < b:
                parts.append((i, a - o, a - p0, b - a))
        out.append((p0, p1 - p0, parts))
    return out


def _ctas(nbytes: int) -> int:
    return max(1, min(CHAN_CTAS, -(-nbytes // 65536)))


def _groups(parts):
    """Launch groups of at most CH_MAX_SEGS segments (both sides split alike)."""
    m = ops._C.CH_MAX_SEGS
    return [parts[i:i + m] for i in range(0, len(parts), m)] or [[]]


class _Stream:
    def __init__(self, device):
        self.device = device
        self.stream = torch.cuda.Stream(device)
        self.status = ops.new_status(device)
        # raised by the host when the peer is declared dead: queued and waiting
        # launches of this link return without touching the peer's memory
        self.abort = torch.zeros(4, dtype=torch.int32).pin_memory()

    def cancel(self) -> None:
        self.abort[0] = 1

    def idle(self) -> bool:
        return self.stream.query()

    def done_event(self):
        ev = torch.cuda.Event()
        ev.record(self.stream)
        return ev


class ChanTx(_Stream):
    def __init__(self, device, ring: int, ready: int, slots: int, slot_bytes: int, credit: torch.Tensor,
                 timeout_s: float):
        super().__init__(device)
        self.ring, self.ready, self.slots, self.slot_bytes = ring, ready, slots, slot_bytes
        self.credit = credit
        self.seq = 0
        self.timeout_s = timeout_s
        self.sent = 0

    def send(self, tensors: Sequence[torch.Tensor], after: Optional[torch.cuda.Event] = None):
        tensors = [t.contiguous() for t in tensors]
        offs, total = _layout(tensors)
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur) if after is None else self.stream.wait_event(after)
        tmo = int(self.timeout_s * 1e9)
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            for _, n, parts in _pieces(offs, total, self.slot_bytes):
                self.seq += 1
                base = self.ring + ((self.seq - 1) % self.slots) * self.slot_bytes
                for gi, grp in enumerate(_groups(parts)):
                    # the slot's previous message must have been copied out first
                    wait = self.credit.data_ptr() if (gi == 0 and self.seq > self.slots) else 0
                    nb = sum(p[3] for p in grp)
                    ops._C.chan_copy([tensors[i].data_ptr() + to for i, to, _, _ in grp], [base + po for _, _, po, _ in grp],
                                     [ln for *_, ln in grp], wait, (self.seq - self.slots) & 0xFFFFFFFF, tmo,
                                     self.ready, 0, 1, 0, _ctas(nb), self.status, self.abort.data_ptr())
                    ops._n()
        for t in tensors:
            t.record_stream(self.stream)
        self.sent += len(tensors)


class ChanRx(_Stream):
    def __init__(self, device, slots: int, slot_bytes: int, timeout_s: float):
        super().__init__(device)
        self.slots, self.slot_bytes = slots, slot_bytes
        # VMM allocations (zero-filled): the sender's mappings of them are
        # released deterministically when either side goes away
        self.ring = shared_empty((slots, slot_bytes), torch.uint8, device)
        self.ready = shared_empty((4,), torch.int32, device)      # [0] ready, [1] CTA counter
        self.credit_addr = 0            # the sender's credit counter (peer mapping)
        self.seq = 0
        self.expected = 0
        self.timeout_s = timeout_s
        self.received = 0

    def recv(self, tensors: Sequence[torch.Tensor]):
        offs, total = _layout(tensors)
        tmo = int(self.timeout_s * 1e9)
        ready, ctr = self.ready.data_ptr(), self.ready.data_ptr() + 4
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            for _, n, parts in _pieces(offs, total, self.slot_bytes):
                self.seq += 1
                groups = _groups(parts)
                for grp in groups:
                    self.expected = (self.expected + _ctas(sum(p[3] for p in grp))) & 0xFFFFFFFF
                base = self.ring.data_ptr() + ((self.seq - 1) % self.slots) * self.slot_bytes
                for gi, grp in enumerate(groups):
                    last = gi == len(groups) - 1
                    nb = sum(p[3] for p in grp)
                    ops._C.chan_copy([base + po for _, _, po, _ in grp], [tensors[i].data_ptr() + to for i, to, _, _ in grp],
                                     [ln for *_, ln in grp], ready, self.expected, tmo,
                                     self.credit_addr if last else 0, self.seq & 0xFFFFFFFF, 2 if last else 0, ctr,
                                     _ctas(nb), self.status, self.abort.data_ptr())
                    ops._n()
        for t in tensors:
            t.record_stream(self.stream)
        self.received += len(tensors)


class ChanLinks:
    """All channels of one endpoint ``me`` (the PairLinks interface)."""

    def __init__(self, store: dist.Store, me: str, device, slots: int = 4, slot_bytes: int = 64 << 20,
                 timeout_s: float = 10.0, wait_s: float = 60.0):
        self.store, self.me = store, me
        self.device = torch.device(device)
        self.slots, self.slot_bytes = slots, slot_bytes
        self.timeout_s, self.wait = timeout_s, timedelta(seconds=wait_s)
        self.mapper = PeerMapper(self.device.index)
        self._links: Dict[Tuple[str, bool], object] = {}
        self._graveyard: List[_Stream] = []    # dropped links whose launches may still be queued
        self._lock = threading.Lock()

    @staticmethod
    def _key(sender: str, receiver: str, what: str) -> str:
        return f"cxch/{sender}>{receiver}/{what}"

    def _get(self, key: str):
        self.store.wait([key], self.wait)
        return pickle.loads(self.store.get(key))

    def open_tx(self, peer: str, gen: int = 0) -> ChanTx:
        with self._lock:
            hit = self._links.get((peer, True))
        if hit is not None:
            return hit
        credit = shared_empty((4,), torch.int32, self.device)
        self.store.set(self._key(self.me, peer, "tx"), pickle.dumps(export_tensor(credit).to_dict()))
        rx = self._get(self._key(self.me, peer, "rx"))
        ring = self.mapper.open(PeerHandle.from_dict(rx["ring"]), owner=peer)
        ready = self.mapper.open(PeerHandle.from_dict(rx["ready"]), owner=peer)
        link = ChanTx(self.device, ring, ready, rx["slots"], rx["slot_bytes"], credit, self.timeout_s)
        with self._lock:
            self._links[(peer, True)] = link
        return link

    def open_rx(self, peer: str, gen: int = 0) -> ChanRx:
        with self._lock:
            hit = self._links.get((peer, False))
        if hit is not None:
            return hit
        link = ChanRx(self.device, self.slots, self.slot_bytes, self.timeout_s)
        self.store.set(self._key(peer, self.me, "rx"), pickle.dumps({
            "ring": export_tensor(link.ring).to_dict(), "ready": export_tensor(link.ready).to_dict(),
            "slots": self.slots, "slot_bytes": self.slot_bytes}))
        tx = self._get(self._key(peer, self.me, "tx"))
        link.credit_addr = self.mapper.open(PeerHandle.from_dict(tx), owner=peer)
        with self._lock:
            self._links[(peer, False)] = link
        return link

    def get(self, peer: str, gen: int = 0, tx: bool = True):
        return self._links.get((peer, tx))

    def drop_peer(self, peer: str, abort: bool = True) -> int:
        """Forget ``peer``'s links.  With ``abort`` their queued and waiting
        launches return at once (status CX_ERR_PEER) instead of waiting out
        their timeout, and store nothing into the peer's memory; the link
        objects stay alive until their streams have drained (their abort
        words and buffers are still read by those launches), and so do the
        mappings of the peer's memory: they are released once those streams
        have passed (:meth:`reap`, also run by :meth:`check`)."""
        with self._lock:
            keys = [k for k in self._links if k[0] == peer]
            dropped = [self._links.pop(k) for k in keys]
            self._graveyard = [l for l in self._graveyard if not l.idle()] + dropped
        if abort:
            for l in dropped:
                l.cancel()
        self.mapper.forget(peer, [l.stream for l in dropped])
        self.mapper.reap()
        return len(keys)

    def reap(self) -> int:
        """Release dropped peers' mappings whose streams have passed; returns
        how many are still held."""
        return self.mapper.reap()

    def check(self) -> None:
        self.mapper.reap()
        for l in list(self._links.values()):
            ops.check_status(l.status, "p2p channel")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self._links.clear()
        self._graveyard.clear()
        self.mapper.close()

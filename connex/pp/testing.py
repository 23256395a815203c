"""Test doubles for the pipeline step protocol (no GPU, no RDMA, no cluster).

:class:`LoopbackTransferEngine`
    an in-process stand-in for a one-sided transfer engine: every engine's
    memory is a set of byte buffers at fake addresses, engines find each
    other by URL in a process-wide table, and ``transfer_sync_read`` copies
    bytes from the named peer's buffer into this engine's.

:class:`FakeLink` / :func:`fake_chain`
    an in-process :class:`connex.pp.hooks.StepTransport` per stage, with the
    endpoint's delivery rules -- replies matched to steps by correlation id
    in any order, duplicates answered from a reply cache, stale ids dropped
    -- and fault knobs on every stage's inbound :class:`Channel`: drop or
    duplicate the next messages, or go dead.  ``fail_over`` reroutes stage 0
    to a new replica; steps sent on the old chain count as lost.

Behavioural parity: ``connex/pp/testing.py:26-218`` of the reference (the
same knobs and rules; the structures are this module's own).
"""
from __future__ import annotations

import bisect
import collections
import threading
import time
from typing import Dict, List, Optional, Set, Tuple

from connex.pp.steps import CorrFilter, ReplyCache, StepIds

_SLOT = 1 << 20      # fake address spacing of loopback buffers


class _Fabric:
    """Process-wide table of loopback engines and the fake address counter."""

    def __init__(self):
        self.lock = threading.Lock()
        self.engines: Dict[str, "LoopbackTransferEngine"] = {}
        self.next_addr = _SLOT

    def take_addresses(self, size: int) -> int:
        with self.lock:
            addr = self.next_addr
            self.next_addr += max(_SLOT, -(-size // _SLOT) * _SLOT)
            return addr


_FABRIC = _Fabric()


class LoopbackTransferEngine:
    """The data-plane surface the PP endpoint uses, over host byte buffers."""

    registry = _FABRIC.engines

    def __init__(self, url: str):
        self.url = url
        self._bases: List[int] = []               # sorted buffer addresses
        self._bufs: Dict[int, bytearray] = {}
        self.reads = 0
        with _FABRIC.lock:
            _FABRIC.engines[url] = self

    @property
    def mem(self) -> Dict[int, bytearray]:
        return self._bufs

    def _locate(self, addr: int, length: int = 1) -> Tuple[bytearray, int]:
        """(buffer, offset) holding ``[addr, addr + length)``; KeyError if none."""
        i = bisect.bisect_right(self._bases, addr) - 1
        if i >= 0:
            base = self._bases[i]
            buf = self._bufs[base]
            if addr + length <= base + max(1, len(buf)):
                return buf, addr - base
        raise KeyError(hex(addr))

    def allocate_managed_buffer(self, size: int) -> int:
        addr = _FABRIC.take_addresses(size)
        bisect.insort(self._bases, addr)
        self._bufs[addr] = bytearray(size)
        return addr

    def free_managed_buffer(self, ptr: int, size: int) -> None:
        if self._bufs.pop(ptr, None) is not None:
            self._bases.remove(ptr)

    def write_bytes_to_buffer(self, ptr: int, data: bytes, length: int) -> None:
        buf, off = self._locate(ptr, length)
        buf[off:off + length] = data[:length]

    def read_bytes_from_buffer(self, ptr: int, length: int) -> bytes:
        buf, off = self._locate(ptr, length)
        return bytes(buf[off:off + length])

    def transfer_sync_read(self, remote_url: str, dst_ptr: int, src_ptr: int, length: int) -> int:
        peer = _FABRIC.engines.get(remote_url)
        if peer is None:
            return -1
        try:
            payload = peer.read_bytes_from_buffer(src_ptr, length)
        except KeyError:
            return -1
        self.write_bytes_to_buffer(dst_ptr, payload, length)
        self.reads += 1
        return 0

    def register_memory(self, ptr: int, length: int) -> int:
        return 0

    def unregister_memory(self, ptr: int) -> int:
        return 0

    def get_rpc_port(self) -> int:
        return 0


class Channel:
    """A stage's inbound message queue with fault knobs: ``drop_next`` /
    ``dup_next`` drop or duplicate that many upcoming messages; a ``dead``
    channel swallows everything."""

    def __init__(self):
        self._items: collections.deque = collections.deque()
        self._cv = threading.Condition()
        self.drop_next = 0
        self.dup_next = 0
        self.dead = False

    def put(self, item) -> None:
        if self.dead:
            return
        if self.drop_next > 0:
            self.drop_next -= 1
            return
        copies = 1
        if self.dup_next > 0:
            self.dup_next -= 1
            copies = 2
        with self._cv:
            self._items.extend([item] * copies)
            self._cv.notify_all()

    def get(self, timeout_s: float):
        """The next message, or None after ``timeout_s`` without one."""
        end = time.monotonic() + max(0.0, timeout_s)
        with self._cv:
            while not self._items:
                left = end - time.monotonic()
                if left <= 0:
                    return None
                self._cv.wait(left)
            return self._items.popleft()


_Wire = Channel     # earlier name of the same class


class FakeLink:
    """One stage of an in-process pipeline.  Stage 0 sends steps downstream;
    every stage forwards to the next and the last one returns to stage 0
    (``head``)."""

    def __init__(self, stage_idx: int, num_stages: int, k: int = 1):
        self.stage_idx, self.num_stages = stage_idx, num_stages
        self.is_first, self.is_last = stage_idx == 0, stage_idx == num_stages - 1
        self._k = k
        self.inbox = Channel()
        self.downstream: Optional[FakeLink] = None
        self.head: Optional[FakeLink] = None
        self.healthy = True
        self.computed = 0
        self.sent = 0
        # stage-0 side: ids awaiting replies, replies that came early, chain epochs
        self.ids = StepIds(0xC0DE << 32)
        self._awaiting: Set[int] = set()
        self._early: Dict[int, dict] = {}
        self.chain_epoch = 0
        self._sent_in: Dict[int, int] = {}
        # forwarding side: stale filter and reply cache for duplicates
        self.filter = CorrFilter(window=k)
        self._cache = ReplyCache(k)

    @property
    def inflight(self) -> int:
        return self._k

    @property
    def outstanding(self) -> Set[int]:
        return self._awaiting

    def _next_hop(self) -> "FakeLink":
        return self.head if self.is_last else self.downstream

    # ---------------------------------------------------------- stage 0
    def new_step_id(self) -> int:
        corr = self.ids.next()
        self._awaiting.add(corr)
        return corr

    def fail_over(self, new_downstream: "FakeLink") -> None:
        """The peer is confirmed dead: route to ``new_downstream``; steps
        sent on the old chain are lost (stale)."""
        self.downstream = new_downstream
        self.chain_epoch += 1

    def step_stale(self, corr: int) -> bool:
        epoch = self._sent_in.get(corr)
        return epoch is not None and epoch != self.chain_epoch

    def send_step(self, td: dict, corr: int, dst=None) -> None:
        self.sent += 1
        self._sent_in[corr] = self.chain_epoch
        self.downstream.inbox.put((corr, dict(td)))

    def recv_step(self, corr: int, timeout_s: Optional[float] = None):
        if corr in self._early:
            self._awaiting.discard(corr)
            return self._early.pop(corr)
        end = time.monotonic() + (0.2 if timeout_s is None else timeout_s)
        while not self.step_stale(corr):
            left = end - time.monotonic()
            if left <= 0:
                return None
            msg = self.inbox.get(min(0.02, left))
            if msg is None:
                continue
            got, td = msg
            if got == corr:
                self._awaiting.discard(corr)
                return td
            if got in self._awaiting:
                self._early[got] = td     # a reply to another in-flight step
        return None

    def abandon_step(self, corr: int) -> None:
        self._awaiting.discard(corr)
        self._early.pop(corr, None)

    def downstream_healthy(self) -> bool:
        d = self.downstream
        return d is not None and d.healthy and not d.inbox.dead

    # ---------------------------------------------------- later stages
    def recv_forward(self, timeout_s: float = 0.2):
        while True:
            msg = self.inbox.get(timeout_s)
            if msg is None:
                return None, None
            corr, td = msg
            cached = self._cache.get(corr)
            if cached is not None:                     # a duplicate: answer it again
                self._next_hop().inbox.put((corr, dict(cached)))
                continue
            if self.filter.accept(corr):
                self.computed += 1
                return td, (corr, None)

    def send_reply(self, td: dict, ctx) -> None:
        corr = ctx[0]
        self._cache.put(corr, dict(td))
        self._next_hop().inbox.put((corr, dict(td)))


def fake_chain(num_stages: int, k: int = 1) -> List[FakeLink]:
    """``num_stages`` linked :class:`FakeLink` objects, stage 0 first."""
    links = [FakeLink(i, num_stages, k) for i in range(num_stages)]
    for here, there in zip(links, links[1:]):
        here.downstream = there
    for link in links:
        link.head = links[0]
    return links

"""Peer memory inside one NVLink/NVSwitch box (one process per GPU).

Two export kinds:

* ``vmm`` -- tensors made by :func:`shared_empty` live in one VMM allocation
  (``cuMemCreate`` with a POSIX-fd handle type, :class:`connex_b200.engine.DeviceBuffer`).
  A peer fetches a duplicate of the allocation's fd over a Unix socket
  (same user only) and maps it.  The physical memory lives until the owner
  *and* every mapping are gone -- so when the owner dies, the peers'
  mappings are all that keep it, and releasing them frees it.
* ``ipc`` -- any other tensor, through the legacy IPC handle of the
  caching-allocator block that contains it plus the tensor's offset.

A peer opens a handle once per allocation (:class:`PeerMapper`) and gets an
address it hands to this package's kernels, which then load from / store to
the owner's HBM over NVLink.  Handles travel over any control channel
(``torch.distributed`` store or object collectives, the ZeroMQ control
plane).

Release is deterministic: :meth:`PeerMapper.forget` moves a peer's mappings
to a :class:`Graveyard` together with an event recorded on every stream that
used them, and :meth:`Graveyard.reap` releases a mapping only after those
events passed -- a kernel still queued against a dead peer's memory never
finds it unmapped, and the memory is freed as soon as nothing can reach it.

Only this package's own kernels are given peer addresses: no library kernel
(GEMM, attention, TMA-multicast code) ever reads another GPU's memory.

Behavioural parity: the "mapping outlives exporter" rule and the deferred
unmap of the reference's ``connex/pd/dataplane.py:46-51`` and
``connex/adapters/vllm/pp/ipcchan.py:283-300``.
"""
from __future__ import annotations

import logging
import math
import os
import threading
import time
import weakref
from dataclasses import dataclass, field
from typing import Callable, Dict, Hashable, Iterable, List, Optional, Tuple

import torch

from connex_b200 import ops

log = logging.getLogger("connex_b200.peer")


@dataclass(frozen=True)
class PeerHandle:
    handle: bytes
    offset: int
    nbytes: int
    owner_device: int
    owner_pid: int
    kind: str = "ipc"                      # "ipc" (legacy handle) or "vmm" (fd of a VMM allocation)
    desc: Optional[dict] = field(default=None, compare=False)   # vmm: DeviceBuffer.describe()

    def to_dict(self) -> dict:
        return {"handle": self.handle, "offset": self.offset, "nbytes": self.nbytes,
                "owner_device": self.owner_device, "owner_pid": self.owner_pid, "kind": self.kind,
                "desc": self.desc}

    @classmethod
    def from_dict(cls, d: dict) -> "PeerHandle":
        return cls(bytes(d["handle"]), int(d["offset"]), int(d["nbytes"]), int(d["owner_device"]),
                   int(d["owner_pid"]), d.get("kind", "ipc"), d.get("desc"))

    @property
    def key(self) -> Hashable:
        """One mapping per allocation."""
        if self.kind == "vmm":
            return ("vmm", self.desc["sock"], int(self.desc["id"]))
        return ("ipc", self.handle)


# ---------------------------------------------------------------- VMM tensors
class _Cuda:
    """``__cuda_array_interface__`` of a DeviceBuffer as bytes; the tensor
    made from it keeps this object (and so the buffer) alive."""

    def __init__(self, buf):
        self.buf = buf
        self.__cuda_array_interface__ = {"shape": (buf.size,), "typestr": "|u1", "data": (buf.ptr, False),
                                         "version": 3, "strides": None, "stream": None}


_SHARED: Dict[int, "weakref.ref[_Cuda]"] = {}
_SHARED_LOCK = threading.Lock()


def shared_empty(shape, dtype: torch.dtype, device) -> torch.Tensor:
    """An uninitialised tensor in its own VMM allocation, exportable to peers
    as a ``vmm`` handle (:func:`export_tensor`)."""
    from connex_b200.engine import DeviceBuffer
    device = torch.device(device)
    nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
    holder = _Cuda(DeviceBuffer(max(nbytes, 1), device.index))
    raw = torch.as_tensor(holder, device=device)
    with _SHARED_LOCK:
        for k in [k for k, r in _SHARED.items() if r() is None]:
            del _SHARED[k]
        _SHARED[holder.buf.ptr] = weakref.ref(holder)
    return raw[:nbytes].view(dtype).view(shape)


def _vmm_owner(ptr: int):
    with _SHARED_LOCK:
        for base, ref in _SHARED.items():
            h = ref()
            if h is not None and base <= ptr < base + h.buf.size:
                return h.buf
    return None


def export_tensor(t: torch.Tensor) -> PeerHandle:
    buf = _vmm_owner(t.data_ptr())
    nbytes = t.numel() * t.element_size()
    if buf is not None:
        return PeerHandle(b"", t.data_ptr() - buf.ptr, nbytes, t.device.index, os.getpid(), "vmm", buf.describe())
    h, off = ops.ipc_export(t.data_ptr(), t.device.index)
    return PeerHandle(h, off, nbytes, t.device.index, os.getpid())


# ------------------------------------------------------------------ graveyard
class Graveyard:
    """Mappings that must not be released yet.  ``passed()`` says whether every
    launch that may touch a mapping has finished; :meth:`reap` releases those
    and keeps the rest."""

    def __init__(self):
        self._graves: List[Tuple[Callable[[], bool], Callable[[], None], int, str]] = []
        self._lock = threading.Lock()
        self.buried = self.released = self.released_bytes = 0

    def bury(self, passed: Callable[[], bool], release: Callable[[], None], nbytes: int = 0, what: str = "") -> None:
        with self._lock:
            self._graves.append((passed, release, nbytes, what))
            self.buried += 1

    def reap(self) -> int:
        """Release what may be released now; returns how many are left."""
        with self._lock:
            ready, keep = [], []
            for g in self._graves:
                (ready if g[0]() else keep).append(g)
            self._graves = keep
        for passed, release, nbytes, what in ready:
            try:
                release()
            except Exception as e:  # noqa: BLE001 - a context already torn down, say
                log.warning("releasing %s failed: %s", what, e)
            with self._lock:
                self.released += 1
                self.released_bytes += nbytes
        return len(self)

    def drain(self, timeout_s: float) -> int:
        end = time.monotonic() + timeout_s
        left = self.reap()
        while left and time.monotonic() < end:
            time.sleep(0.001)
            left = self.reap()
        return left

    def __len__(self) -> int:
        with self._lock:
            return len(self._graves)


class _Open:
    __slots__ = ("base", "nbytes", "owner", "mapping", "kind")

    def __init__(self, base, nbytes, owner, mapping, kind):
        self.base, self.nbytes, self.owner, self.mapping, self.kind = base, nbytes, owner, mapping, kind


class PeerMapper:
    """Opens peer handles (once per allocation) and releases them
    deterministically: :meth:`forget` (a peer that left or died) buries its
    mappings until the streams that used them have passed; :meth:`close`
    releases everything."""

    def __init__(self, device: int, graveyard: Optional[Graveyard] = None):
        self.device = device
        self._open: Dict[Hashable, _Open] = {}
        self.graveyard = graveyard if graveyard is not None else Graveyard()
        self._lock = threading.Lock()

    def open(self, h: PeerHandle, owner: Optional[Hashable] = None) -> int:
        """Local address of ``h``'s first byte; ``owner`` (default: the
        exporting pid) groups mappings for :meth:`forget`."""
        if h.owner_pid == os.getpid():
            raise ValueError("handle belongs to this process; use the local address")
        with self._lock:
            o = self._open.get(h.key)
            if o is None:
                if h.kind == "vmm":
                    from connex_b200.engine import Mapping
                    m = Mapping(h.desc, self.device)
                    o = _Open(m.ptr, int(h.desc["alloc_size"]), owner if owner is not None else h.owner_pid, m,
                              "vmm")
                else:
                    base = ops.ipc_open(h.handle, self.device)
                    o = _Open(base, h.offset + h.nbytes, owner if owner is not None else h.owner_pid, None, "ipc")
                self._open[h.key] = o
        return o.base + h.offset

    def owners(self) -> List[Hashable]:
        with self._lock:
            return sorted({o.owner for o in self._open.values()}, key=str)

    def _release_fn(self, o: _Open) -> Callable[[], None]:
        if o.kind == "vmm":
            return o.mapping.release
        dev = self.device
        return lambda: ops.ipc_close(o.base, dev)

    def _passed_fn(self, o: _Open, streams: List, fences: List) -> Callable[[], bool]:
        checks = [f.query for f in fences]
        if streams and o.kind == "vmm":
            for s in streams:
                o.mapping.record(s.cuda_stream)
            checks.append(o.mapping.passed)
        elif streams:
            for s in streams:
                e = torch.cuda.Event()
                e.record(s)
                checks.append(e.query)
        return lambda: all(c() for c in checks)

    def forget(self, owner: Hashable, streams: Iterable = (), fences: Iterable = ()) -> int:
        """Bury ``owner``'s mappings; each is released once everything queued
        so far on ``streams`` (the streams whose launches used it) has
        finished and every fence (anything with ``query()``, e.g. an event
        the caller recorded) has passed.  Returns how many were buried."""
        streams, fences = list(streams), list(fences)
        with self._lock:
            gone = [(k, o) for k, o in self._open.items() if o.owner == owner]
            for k, _ in gone:
                del self._open[k]
        for _, o in gone:
            self.graveyard.bury(self._passed_fn(o, streams, fences), self._release_fn(o), o.nbytes,
                                f"{o.kind} of {owner}")
        return len(gone)

    def reap(self) -> int:
        return self.graveyard.reap()

    def close(self, timeout_s: float = 10.0) -> int:
        """Release every mapping (after the device's queued work passed);
        returns how many are still held (kept rather than unmapped in use)."""
        if torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
        for owner in self.owners():
            self.forget(owner)
        left = self.graveyard.drain(timeout_s)
        if left:
            log.warning("%d peer mapping(s) still in use after %.1f s: kept", left, timeout_s)
        return left


def enable_all_peers(device: int, world: int) -> None:
    for p in range(world):
        if p != device:
            try:
                ops.enable_peer_access(device, p)
            except RuntimeError:
                pass

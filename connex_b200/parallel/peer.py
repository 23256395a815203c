"""Peer memory inside one NVLink/NVSwitch box (one process per GPU).

A buffer is exported as a CUDA IPC handle of the allocation that contains it
plus the buffer's offset inside that allocation; a peer process opens the
handle once and gets an address it can hand to this package's kernels, which
then load from / store to the owner's HBM over NVLink.  Handles travel over
any control channel (``torch.distributed`` object collectives here, or the
ZeroMQ control plane).

Only this package's own kernels are given peer addresses: no library kernel
(GEMM, attention, TMA-multicast code) ever reads another GPU's memory.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

from connex_b200 import ops


@dataclass(frozen=True)
class PeerHandle:
    handle: bytes
    offset: int
    nbytes: int
    owner_device: int
    owner_pid: int

    def to_dict(self) -> dict:
        return {"handle": self.handle, "offset": self.offset, "nbytes": self.nbytes,
                "owner_device": self.owner_device, "owner_pid": self.owner_pid}

    @classmethod
    def from_dict(cls, d: dict) -> "PeerHandle":
        return cls(bytes(d["handle"]), int(d["offset"]), int(d["nbytes"]), int(d["owner_device"]),
                   int(d["owner_pid"]))


def export_tensor(t: torch.Tensor) -> PeerHandle:
    import os
    h, off = ops.ipc_export(t.data_ptr(), t.device.index)
    return PeerHandle(h, off, t.numel() * t.element_size(), t.device.index, os.getpid())


class PeerMapper:
    """Opens peer handles (once per allocation) and closes them on ``close()``."""

    def __init__(self, device: int):
        self.device = device
        self._open: Dict[bytes, int] = {}

    def open(self, h: PeerHandle) -> int:
        import os
        if h.owner_pid == os.getpid():
            raise ValueError("handle belongs to this process; use the local address")
        base = self._open.get(h.handle)
        if base is None:
            base = ops.ipc_open(h.handle, self.device)
            self._open[h.handle] = base
        return base + h.offset

    def close(self) -> None:
        for base in self._open.values():
            try:
                ops.ipc_close(base, self.device)
            except RuntimeError:
                pass
        self._open.clear()


def enable_all_peers(device: int, world: int) -> None:
    for p in range(world):
        if p != device:
            try:
                ops.enable_peer_access(device, p)
            except RuntimeError:
                pass

"""Pinned host mirror of registered KV spans, for data planes that cannot
reach GPU memory (no peer-memory driver, or the TCP engine between hosts).

Producer: after the prefill that wrote a request's blocks, ``stage_out``
copies them into the pinned mirror on the engine stream and returns an
event; the control reply that hands the blocks to a reader waits for it.
Readers read the mirror.  Consumer: a pull reads into its own mirror and
``stage_in`` copies what arrived back to the device on a side stream that is
ordered after the engine stream.

``CONNEX_PD_HOST_STAGING`` = ``auto`` (default: stage only when the plane
refuses device memory) | ``1`` (always) | ``0`` (never).
Behavioural parity: ``connex/pd/host_staging.py:36-196`` of the reference.
"""
from __future__ import annotations

import bisect
import logging
import os
from dataclasses import dataclass, replace
from typing import Any, Iterable, List, Optional, Sequence, Tuple

log = logging.getLogger("connex.pd")

_PEERMEM_PATHS = ("/sys/module/nvidia_peermem", "/sys/module/nv_peer_mem", "/sys/kernel/mm/memory_peers/nv_mem")
_TRUTHY = {"true": "1", "yes": "1", "on": "1", "false": "0", "no": "0", "off": "0"}


def gpudirect_available() -> bool:
    """A peer-memory kernel module (GPUDirect RDMA) is loaded."""
    return any(os.path.exists(p) for p in _PEERMEM_PATHS)


def staging_mode() -> str:
    raw = (os.getenv("CONNEX_PD_HOST_STAGING") or "auto").strip().lower()
    return _TRUTHY.get(raw, raw)


@dataclass
class _Mirror:
    start: int          # device address of the span
    length: int
    device: Any         # uint8 view of the device span
    host: Any           # pinned uint8 mirror

    def host_addr(self, addr: int) -> int:
        return self.host.data_ptr() + (addr - self.start)


def merge_ranges(ranges: Iterable[Tuple[int, int]]) -> List[Tuple[int, int]]:
    """Sorted (address, length) ranges with touching or overlapping ones joined."""
    joined: List[List[int]] = []
    for a, n in sorted(ranges):
        if joined and a <= joined[-1][1]:
            joined[-1][1] = max(joined[-1][1], a + n)
        else:
            joined.append([a, a + n])
    return [(a, b - a) for a, b in joined]


class HostStaging:
    def __init__(self, spans: Sequence[Tuple[int, int]], device: Optional[int] = None):
        import torch
        from connex_b200 import ops
        self.torch = torch
        self.device = torch.cuda.current_device() if device is None else device
        self._mirrors = [_Mirror(s, n, ops.from_ptr(s, [n], torch.uint8, self.device),
                                 torch.empty(n, dtype=torch.uint8, pin_memory=True))
                         for s, n in sorted(spans)]
        self._starts = [m.start for m in self._mirrors]
        self._side = torch.cuda.Stream(device=self.device)
        self._engine = torch.cuda.current_stream(self.device)

    def _mirror_of(self, addr: int) -> _Mirror:
        i = bisect.bisect_right(self._starts, addr) - 1
        if i >= 0 and addr < self._mirrors[i].start + self._mirrors[i].length:
            return self._mirrors[i]
        raise ValueError(f"{addr:#x} is not in a staged KV span")

    def mirror(self, addr: int) -> int:
        """Host address that mirrors device address ``addr``."""
        return self._mirror_of(addr).host_addr(addr)

    def mirror_spans(self) -> List[Tuple[int, int]]:
        return [(m.host.data_ptr(), m.length) for m in self._mirrors]

    def translate(self, layout):
        """The layout as seen in the mirror (what readers must read)."""
        return replace(layout, base=self.mirror(layout.base))

    def mirror_ops(self, ops):
        """Reads retargeted from device destinations to their mirror."""
        return [(self.mirror(d), s, n) for d, s, n in ops]

    def _copy(self, ranges, to_host: bool) -> None:
        for addr, n in merge_ranges(ranges):
            m = self._mirror_of(addr)
            o = addr - m.start
            dst, src = (m.host, m.device) if to_host else (m.device, m.host)
            dst[o:o + n].copy_(src[o:o + n], non_blocking=True)

    def stage_out(self, ranges):
        """Device -> mirror on the current (engine) stream; returns its event."""
        torch = self.torch
        with torch.cuda.device(self.device):
            self._copy(ranges, to_host=True)
            done = torch.cuda.Event()
            done.record()
        return done

    def stage_in(self, ranges) -> None:
        """Mirror -> device on the side stream, after the engine stream's work; waits."""
        torch = self.torch
        with torch.cuda.device(self.device), torch.cuda.stream(self._side):
            self._side.wait_stream(self._engine)
            self._copy(ranges, to_host=False)
        self._side.synchronize()


def block_ranges(layouts, blocks: Sequence[int]) -> List[Tuple[int, int]]:
    """(address, length) of every segment of the given blocks."""
    return [(lo.base + o * lo.outer_stride + b * lo.block_stride, lo.seg_bytes)
            for lo in layouts for o in range(lo.outer) for b in blocks]


def _register_device_spans(plane, spans) -> Optional[Tuple[int, int, int]]:
    """Register every span; on a refusal undo the earlier ones and return
    (start, length, rc) of the refused span."""
    done = []
    for start, n in spans:
        rc = plane.register(start, n)
        if rc != 0:
            for s in done:
                plane.unregister(s)
            return start, n, rc
        done.append(start)
    return None


def register_with_staging(plane, spans, what: str) -> Optional[HostStaging]:
    """Register ``spans`` with ``plane``.  Returns None when the plane took
    the device memory itself; otherwise (forced, or the plane refused device
    memory) registers pinned mirrors and returns the :class:`HostStaging`."""
    from connex.pd.dataplane import is_device_ptr
    mode = staging_mode()
    on_device = bool(spans) and is_device_ptr(spans[0][0])
    if mode == "auto" and on_device and plane.name == "cxengine":
        mode = "1"                          # the TCP engine plane reads host memory only
    if mode != "1":
        refused = _register_device_spans(plane, spans)
        if refused is None:
            return None
        start, n, rc = refused
        if mode == "0" or not is_device_ptr(start):
            raise RuntimeError(f"{plane.name}: register_memory({start:#x}, {n}) = {rc}")
        log.warning("%s: %s cannot register GPU memory (rc %d): staging through host memory", what, plane.name, rc)
    staging = HostStaging(spans)
    for start, n in staging.mirror_spans():
        rc = plane.register(start, n)
        if rc != 0:
            raise RuntimeError(f"{plane.name}: register_memory(host {start:#x}, {n}) = {rc}")
    plane._connex_staging = staging
    return staging

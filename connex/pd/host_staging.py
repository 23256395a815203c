"""Pinned host mirror of registered KV spans (reference ``connex/pd/host_staging.py``).

For data planes that cannot reach GPU memory (no peer-memory driver, or a
TCP plane between hosts): the producer copies held blocks into a pinned
mirror on the engine stream after the prefill that wrote them (``stage_out``
returns an event the control reply waits for), readers read the mirror, and
the consumer copies what it read back to the device on a side stream ordered
after the engine stream (``stage_in``).  ``CONNEX_PD_HOST_STAGING`` =
``auto`` (default) | ``1`` | ``0``.
"""
from __future__ import annotations

import bisect
import logging
import os
from dataclasses import replace
from typing import List, Optional, Sequence, Tuple

log = logging.getLogger("connex.pd")


def gpudirect_available() -> bool:
    return any(os.path.exists(p) for p in ("/sys/module/nvidia_peermem", "/sys/module/nv_peer_mem",
                                           "/sys/kernel/mm/memory_peers/nv_mem"))


def staging_mode() -> str:
    m = (os.getenv("CONNEX_PD_HOST_STAGING") or "auto").strip().lower()
    return {"true": "1", "yes": "1", "on": "1", "false": "0", "no": "0", "off": "0"}.get(m, m)


class HostStaging:
    def __init__(self, spans: Sequence[Tuple[int, int]], device: Optional[int] = None):
        import torch
        from connex_b200 import ops
        self.torch = torch
        self.device = torch.cuda.current_device() if device is None else device
        self._starts: List[int] = []
        self._spans: list = []
        for start, n in sorted(spans):
            dev = ops.from_ptr(start, [n], torch.uint8, self.device)
            mirror = torch.empty(n, dtype=torch.uint8, pin_memory=True)
            self._starts.append(start)
            self._spans.append((start, n, dev, mirror))
        self._stream = torch.cuda.Stream(device=self.device)
        self._engine_stream = torch.cuda.current_stream(self.device)

    def _find(self, addr: int):
        i = bisect.bisect_right(self._starts, addr) - 1
        if i < 0 or addr >= self._spans[i][0] + self._spans[i][1]:
            raise ValueError(f"{addr:#x} is not in a staged KV span")
        start, _, dev, mirror = self._spans[i]
        return start, dev, mirror

    def mirror(self, addr: int) -> int:
        start, _, m = self._find(addr)
        return m.data_ptr() + (addr - start)

    def mirror_spans(self) -> List[Tuple[int, int]]:
        return [(m.data_ptr(), n) for _, n, _, m in self._spans]

    def translate(self, layout):
        return replace(layout, base=self.mirror(layout.base))

    def mirror_ops(self, ops):
        return [(self.mirror(d), s, n) for d, s, n in ops]

    def _copy(self, ranges, to_host: bool) -> None:
        for addr, n in merge_ranges(ranges):
            start, dev, m = self._find(addr)
            o = addr - start
            if to_host:
                m[o:o + n].copy_(dev[o:o + n], non_blocking=True)
            else:
                dev[o:o + n].copy_(m[o:o + n], non_blocking=True)

    def stage_out(self, ranges):
        torch = self.torch
        with torch.cuda.device(self.device):
            self._copy(ranges, to_host=True)
            ev = torch.cuda.Event()
            ev.record()
        return ev

    def stage_in(self, ranges) -> None:
        torch = self.torch
        with torch.cuda.device(self.device), torch.cuda.stream(self._stream):
            self._stream.wait_stream(self._engine_stream)
            self._copy(ranges, to_host=False)
        self._stream.synchronize()


def merge_ranges(ranges) -> List[Tuple[int, int]]:
    out: List[Tuple[int, int]] = []
    for a, n in sorted(ranges):
        if out and a <= out[-1][0] + out[-1][1]:
            pa, pn = out[-1]
            out[-1] = (pa, max(pa + pn, a + n) - pa)
        else:
            out.append((a, n))
    return out


def block_ranges(layouts, blocks: Sequence[int]) -> List[Tuple[int, int]]:
    out = []
    for lo in layouts:
        for o in range(lo.outer):
            b0 = lo.base + o * lo.outer_stride
            out.extend((b0 + b * lo.block_stride, lo.seg_bytes) for b in blocks)
    return out


def register_with_staging(plane, spans, what: str) -> Optional[HostStaging]:
    """Register ``spans`` with ``plane``; stage through pinned host memory when
    the plane cannot reach device memory (or when forced)."""
    from connex.pd.dataplane import is_device_ptr
    mode = staging_mode()
    if mode == "auto" and spans and plane.name == "cxengine" and is_device_ptr(spans[0][0]):
        mode = "1"  # the TCP engine plane reads host memory only
    if mode != "1":
        done = []
        for start, n in spans:
            rc = plane.register(start, n)
            if rc != 0:
                for s in done:
                    plane.unregister(s)
                if mode == "0" or not is_device_ptr(start):
                    raise RuntimeError(f"{plane.name}: register_memory({start:#x}, {n}) = {rc}")
                log.warning("%s: %s cannot register GPU memory (rc %d): staging through host memory",
                            what, plane.name, rc)
                break
            done.append(start)
        else:
            return None
    staging = HostStaging(spans)
    for start, n in staging.mirror_spans():
        rc = plane.register(start, n)
        if rc != 0:
            raise RuntimeError(f"{plane.name}: register_memory(host {start:#x}, {n}) = {rc}")
    plane._connex_staging = staging
    return staging

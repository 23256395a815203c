"""Flat weight arena: every tensor of one model version packed into one
256-byte-aligned byte buffer described by a manifest (reference
``connex/rl/weights.py``).  One buffer = one registration and large one-sided
reads; the manifest rebuilds ``(name, tensor)`` views without copies.
Manifest wire form: ``{"version", "total", "entries": [[name, dtype, shape,
offset, nbytes], ...]}``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable, List, Optional, Tuple

import torch

ALIGN = 256


def _dtype(name: str) -> torch.dtype:
    return getattr(torch, name.replace("torch.", ""))


@dataclass
class TensorEntry:
    name: str
    dtype: str
    shape: list
    offset: int
    nbytes: int


@dataclass
class WeightManifest:
    version: int
    entries: List[TensorEntry] = field(default_factory=list)
    total: int = 0

    def to_dict(self) -> dict:
        return {"version": self.version, "total": self.total,
                "entries": [[e.name, e.dtype, list(e.shape), e.offset, e.nbytes] for e in self.entries]}

    @classmethod
    def from_dict(cls, d: dict) -> "WeightManifest":
        return cls(d["version"], [TensorEntry(*e) for e in d["entries"]], d["total"])

    @classmethod
    def build(cls, version: int, named: Iterable[Tuple[str, torch.Tensor]]) -> "WeightManifest":
        m, off = cls(version), 0
        for name, t in named:
            n = t.numel() * t.element_size()
            m.entries.append(TensorEntry(name, str(t.dtype).replace("torch.", ""), list(t.shape), off, n))
            off += -(-n // ALIGN) * ALIGN
        m.total = max(off, ALIGN)
        return m

    def same_layout(self, other: Optional["WeightManifest"]) -> bool:
        return other is not None and self.total == other.total and \
            [(e.name, e.dtype, e.shape, e.offset) for e in self.entries] == \
            [(e.name, e.dtype, e.shape, e.offset) for e in other.entries]

    def entry(self, name: str) -> TensorEntry:
        for e in self.entries:
            if e.name == name:
                return e
        raise KeyError(name)


def arena_size(named) -> int:
    return WeightManifest.build(0, named).total


def pack_into(arena: torch.Tensor, manifest: WeightManifest, named) -> None:
    """Copy tensors into the uint8 ``arena`` at the manifest's offsets."""
    by = {e.name: e for e in manifest.entries}
    for name, t in named:
        e = by[name]
        arena[e.offset:e.offset + e.nbytes].copy_(t.detach().contiguous().view(-1).view(torch.uint8),
                                                  non_blocking=True)


def unpack(arena: torch.Tensor, manifest: WeightManifest):
    """``(name, tensor)`` views into ``arena`` (no copy)."""
    for e in manifest.entries:
        yield e.name, arena[e.offset:e.offset + e.nbytes].view(_dtype(e.dtype)).view(e.shape)

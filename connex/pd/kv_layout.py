"""Where the bytes of a KV block live, for any paged KV cache (torch-free).

An engine's KV cache is a list of tensors with a ``num_blocks`` dimension;
block ``b`` of a tensor is ``outer`` equally spaced contiguous segments (e.g.
K and V of a ``[2, num_blocks, ...]`` cache).  :class:`TensorLayout` reduces a
tensor to plain numbers that travel between instances; ``read_ops`` turns
(local block, remote block) pairs into the fewest one-sided reads (runs of
consecutive blocks on both sides become one read per segment);
``tp_plan`` / ``head_read_ops`` re-lay KV heads between instances sharded
with different tensor-parallel degrees.  Same semantics and dict format as
the reference's ``connex/pd/kv_layout.py:24-306`` (the layouts travel in the
producer's ``meta`` reply).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, replace
from typing import Iterable, List, Optional, Sequence, Tuple


@dataclass(frozen=True)
class TensorLayout:
    """Block b, segment o starts at ``base + o*outer_stride + b*block_stride``
    and is ``seg_bytes`` long.  Optional head geometry inside a segment: head
    h, token t starts at ``h*head_stride + t*token_stride``, ``head_bytes`` long."""

    base: int
    outer: int
    outer_stride: int
    block_stride: int
    seg_bytes: int
    num_blocks: int
    heads: int = 0
    head_stride: int = 0
    tokens: int = 0
    token_stride: int = 0
    head_bytes: int = 0

    @property
    def span(self) -> Tuple[int, int]:
        end = self.base + (self.outer - 1) * self.outer_stride + self.num_blocks * self.block_stride
        return self.base, end - self.base

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "TensorLayout":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})

    def with_heads(self, heads: int, head_stride: int, tokens: int, token_stride: int,
                   head_bytes: int) -> "TensorLayout":
        if heads * tokens * head_bytes != self.seg_bytes:
            raise ValueError(f"{heads} heads x {tokens} tokens x {head_bytes} B != segment of "
                             f"{self.seg_bytes} B")
        return replace(self, heads=heads, head_stride=head_stride, tokens=tokens, token_stride=token_stride,
                       head_bytes=head_bytes)

    @property
    def head_major(self) -> bool:
        """All tokens of one head are contiguous (HND)."""
        return self.token_stride == self.head_bytes and self.head_stride == self.tokens * self.head_bytes


def _dense(shape: Sequence[int], stride: Sequence[int]) -> bool:
    """The dims cover one dense run of memory in some order."""
    expect = 1
    for s, n in sorted((s, n) for n, s in zip(shape, stride) if n != 1):
        if s != expect:
            return False
        expect *= n
    return True


def tensor_layout(t, num_blocks: int, heads_dims: Optional[Tuple[int, int]] = None) -> TensorLayout:
    """Layout of a tensor whose first ``num_blocks``-sized dimension with a
    dense per-block slice indexes blocks (``[2, nb, ...]`` or ``[nb, ...]``)."""
    shape, stride, es = tuple(t.shape), tuple(t.stride()), t.element_size()
    for d, n in enumerate(shape):
        if n != num_blocks:
            continue
        inner = 1
        for x in shape[d + 1:]:
            inner *= x
        if not (inner and _dense(shape[d + 1:], stride[d + 1:]) and stride[d] >= inner):
            continue
        outer = 1
        for x in shape[:d]:
            outer *= x
        if outer > 1 and d != 1:
            continue
        lo = TensorLayout(base=t.data_ptr(), outer=outer, outer_stride=stride[0] * es if outer > 1 else 0,
                          block_stride=stride[d] * es, seg_bytes=inner * es, num_blocks=num_blocks)
        if heads_dims is not None:
            td, hd = (x % len(shape) for x in heads_dims)
            hb = es
            for x in shape[max(td, hd) + 1:]:
                hb *= x
            lo = lo.with_heads(shape[hd], stride[hd] * es, shape[td], stride[td] * es, hb)
        return lo
    raise ValueError(f"no contiguous num_blocks={num_blocks} dimension in shape {shape} stride {stride}")


def find_heads_dims(shape: tuple, num_blocks: int, kv_heads: int, block_size: int,
                    layout: Optional[str] = None) -> Optional[Tuple[int, int]]:
    """(token dim, head dim) after the block dim, matched by size; when the
    head count equals the block size the layout name (``LBHNC`` = heads
    first, ``LBNHC`` = tokens first) decides."""
    try:
        b = list(shape).index(num_blocks)
    except ValueError:
        return None
    inner = list(range(b + 1, len(shape) - 1))
    hs = [d for d in inner if shape[d] == kv_heads]
    ts = [d for d in inner if shape[d] == block_size]
    if not kv_heads or not hs or not ts:
        return None
    if kv_heads != block_size:
        return ts[0], hs[0]
    if len(inner) < 2:
        return None
    first, second = inner[0], inner[1]
    name = (layout or "").upper()
    if "H" in name and "N" in name and name.index("H") < name.index("N"):
        return second, first
    return first, second


def block_runs(local: Sequence[int], remote: Sequence[int]) -> List[Tuple[int, int, int]]:
    """Coalesce aligned block lists into (local_start, remote_start, count)."""
    if len(local) != len(remote):
        raise ValueError(f"block lists differ in length: {len(local)} vs {len(remote)}")
    runs: List[Tuple[int, int, int]] = []
    for lb, rb in zip(local, remote):
        if runs and lb == runs[-1][0] + runs[-1][2] and rb == runs[-1][1] + runs[-1][2]:
            runs[-1] = (runs[-1][0], runs[-1][1], runs[-1][2] + 1)
        else:
            runs.append((lb, rb, 1))
    return runs


def read_ops(local_layouts: Sequence[TensorLayout], remote_layouts: Sequence[TensorLayout],
             local_blocks: Sequence[int], remote_blocks: Sequence[int]) -> List[Tuple[int, int, int]]:
    """(dst, src, length) reads copying the peer's ``remote_blocks`` into ours."""
    if len(local_layouts) != len(remote_layouts):
        raise ValueError(f"peer has {len(remote_layouts)} KV tensors, we have {len(local_layouts)}")
    runs = block_runs(local_blocks, remote_blocks)
    ops = []
    for lo, ro in zip(local_layouts, remote_layouts):
        if (lo.seg_bytes, lo.outer) != (ro.seg_bytes, ro.outer):
            raise ValueError(f"KV layout mismatch between instances (segment {lo.seg_bytes} vs {ro.seg_bytes} "
                             f"bytes, {lo.outer} vs {ro.outer} segments per block)")
        dense = lo.block_stride == lo.seg_bytes and ro.block_stride == ro.seg_bytes
        for o in range(lo.outer):
            lb, rb = lo.base + o * lo.outer_stride, ro.base + o * ro.outer_stride
            for l0, r0, n in runs:
                if dense:
                    ops.append((lb + l0 * lo.block_stride, rb + r0 * ro.block_stride, n * lo.seg_bytes))
                else:
                    ops.extend((lb + (l0 + i) * lo.block_stride, rb + (r0 + i) * ro.block_stride, lo.seg_bytes)
                               for i in range(n))
    return ops


def register_spans(layouts: Iterable[TensorLayout]) -> List[Tuple[int, int]]:
    """Distinct memory spans to register, merged only where they overlap."""
    out: List[Tuple[int, int]] = []
    for s, n in sorted(lo.span for lo in layouts):
        if out and s < out[-1][0] + out[-1][1]:
            ps, pn = out[-1]
            out[-1] = (ps, max(ps + pn, s + n) - ps)
        else:
            out.append((s, n))
    return out


@dataclass(frozen=True)
class TPSource:
    """A remote TP rank this local rank reads: ``nheads`` heads from remote
    head ``remote_head0`` to local head ``local_head0`` (rank-relative);
    ``readers`` local ranks read it and the lowest is its ``releaser``."""

    remote_rank: int
    nheads: int
    local_head0: int
    remote_head0: int
    releaser: bool
    readers: int


def tp_plan(local_rank: int, local_tp: int, remote_tp: int, total_heads: int) -> List[TPSource]:
    """Sources of local rank ``local_rank`` when KV heads are sharded
    contiguously (rank r holds heads [r*H/tp, (r+1)*H/tp))."""
    for tp in (local_tp, remote_tp):
        if tp < 1 or total_heads % tp:
            raise ValueError(f"{total_heads} KV heads cannot be sharded over TP {tp} "
                             "(replicated KV heads are not supported)")
    if not 0 <= local_rank < local_tp:
        raise ValueError(f"rank {local_rank} outside TP {local_tp}")
    hl, hr = total_heads // local_tp, total_heads // remote_tp
    lo, hi = local_rank * hl, (local_rank + 1) * hl
    out = []
    for p in range(lo // hr, -(-hi // hr)):
        a, b = max(lo, p * hr), min(hi, (p + 1) * hr)
        first_reader, last_reader = (p * hr) // hl, ((p + 1) * hr - 1) // hl
        out.append(TPSource(p, b - a, a - lo, a - p * hr, local_rank == first_reader,
                            last_reader - first_reader + 1))
    return out


def _append_merged(ops: list, dst: int, src: int, n: int) -> None:
    if ops and ops[-1][0] + ops[-1][2] == dst and ops[-1][1] + ops[-1][2] == src:
        ops[-1] = (ops[-1][0], ops[-1][1], ops[-1][2] + n)
    else:
        ops.append((dst, src, n))


def head_read_ops(local_layouts: Sequence[TensorLayout], remote_layouts: Sequence[TensorLayout],
                  local_blocks: Sequence[int], remote_blocks: Sequence[int], local_head0: int,
                  remote_head0: int, nheads: int) -> List[Tuple[int, int, int]]:
    """Reads copying remote heads [remote_head0, +nheads) of the peer's blocks
    into local heads [local_head0, +nheads) (HND or NHD on either side)."""
    if len(local_layouts) != len(remote_layouts):
        raise ValueError(f"peer has {len(remote_layouts)} KV tensors, we have {len(local_layouts)}")
    runs = block_runs(local_blocks, remote_blocks)
    ops: list = []
    for lo, ro in zip(local_layouts, remote_layouts):
        if not (lo.heads and ro.heads):
            raise ValueError("KV head geometry unknown: cannot re-layout heads")
        if (lo.tokens, lo.head_bytes, lo.outer) != (ro.tokens, ro.head_bytes, ro.outer):
            raise ValueError("KV layout mismatch between instances (block tokens / head bytes / segments)")
        if local_head0 + nheads > lo.heads or remote_head0 + nheads > ro.heads:
            raise ValueError(f"head range outside the shard ({local_head0}+{nheads} of {lo.heads} local, "
                             f"{remote_head0}+{nheads} of {ro.heads} remote)")
        if lo.head_major and ro.head_major:
            pieces = [(local_head0 * lo.head_stride, remote_head0 * ro.head_stride, nheads * lo.head_stride)]
        elif lo.head_stride == lo.head_bytes and ro.head_stride == ro.head_bytes:
            pieces = [(t * lo.token_stride + local_head0 * lo.head_bytes,
                       t * ro.token_stride + remote_head0 * ro.head_bytes, nheads * lo.head_bytes)
                      for t in range(lo.tokens)]
        else:
            pieces = [((local_head0 + h) * lo.head_stride + t * lo.token_stride,
                       (remote_head0 + h) * ro.head_stride + t * ro.token_stride, lo.head_bytes)
                      for h in range(nheads) for t in range(lo.tokens)]
        for o in range(lo.outer):
            lb, rb = lo.base + o * lo.outer_stride, ro.base + o * ro.outer_stride
            for l0, r0, n in runs:
                for i in range(n):
                    ld, rs = lb + (l0 + i) * lo.block_stride, rb + (r0 + i) * ro.block_stride
                    for lo_off, ro_off, ln in pieces:
                        _append_merged(ops, ld + lo_off, rs + ro_off, ln)
    return ops


def cx_cache_layouts(kv) -> List[TensorLayout]:
    """Layouts of a connex_b200 paged cache ``[L, 2, blocks, Hkv, BS, D]``: one
    layout per layer with K and V as the two segments, head geometry HND."""
    L, _, nb, H, BS, D = kv.shape
    es = kv.element_size()
    st = kv.stride()
    out = []
    for l in range(L):
        lo = TensorLayout(base=kv.data_ptr() + l * st[0] * es, outer=2, outer_stride=st[1] * es,
                          block_stride=st[2] * es, seg_bytes=H * BS * D * es, num_blocks=nb)
        out.append(lo.with_heads(H, st[3] * es, BS, st[4] * es, D * es))
    return out

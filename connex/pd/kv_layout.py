"""Where the bytes of a KV block live, for any paged KV cache (torch-free).

An engine's KV cache is a list of tensors with a ``num_blocks`` dimension;
block ``b`` of one tensor is ``outer`` equally spaced contiguous segments
(K and V of a ``[2, num_blocks, ...]`` cache are two segments).
:class:`TensorLayout` reduces such a tensor to numbers that travel between
instances (the producer's ``meta`` reply carries them as dicts), and the
functions here turn them into one-sided reads:

* :func:`read_ops` -- copy whole blocks; runs of consecutive blocks on both
  sides become one read per segment when blocks are densely packed;
* :func:`tp_plan` / :func:`head_read_ops` -- copy a range of KV heads between
  instances sharded over different tensor-parallel degrees, for head-major
  (HND) or token-major (NHD) blocks on either side.

The dict format and the semantics match ``connex/pd/kv_layout.py:24-306`` of
the reference (layouts of either implementation can be exchanged).
"""
from __future__ import annotations

import itertools
from dataclasses import asdict, dataclass, fields, replace
from math import prod
from typing import Iterable, Iterator, List, Optional, Sequence, Tuple

Op = Tuple[int, int, int]            # (dst address, src address, bytes)


@dataclass(frozen=True)
class TensorLayout:
    """Segment ``o`` of block ``b`` starts at ``base + o*outer_stride +
    b*block_stride`` and is ``seg_bytes`` long.  Optional head geometry in a
    segment: head ``h`` of token ``t`` starts at ``h*head_stride +
    t*token_stride`` and is ``head_bytes`` long."""

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

    def segment(self, o: int, b: int) -> int:
        return self.base + o * self.outer_stride + b * self.block_stride

    @property
    def span(self) -> Tuple[int, int]:
        """(start, length) of the memory this tensor's blocks occupy."""
        end = self.segment(self.outer - 1, self.num_blocks)
        return self.base, end - self.base

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "TensorLayout":
        names = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in names})

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

    @property
    def token_major(self) -> bool:
        """All heads of one token are contiguous (NHD)."""
        return self.head_stride == self.head_bytes


def _packed(shape: Sequence[int], stride: Sequence[int]) -> bool:
    """True when the (size > 1) dims tile one dense run of memory, in any order."""
    dims = sorted((st, n) for n, st in zip(shape, stride) if n != 1)
    covered = 1
    for st, n in dims:
        if st != covered:
            return False
        covered *= n
    return True


def tensor_layout(t, num_blocks: int, heads_dims: Optional[Tuple[int, int]] = None) -> TensorLayout:
    """Layout of a tensor indexed by blocks in its first ``num_blocks``-sized
    dimension whose per-block slice is dense (``[nb, ...]`` or ``[2, nb, ...]``).
    ``heads_dims`` = (token dim, head dim) adds the head geometry."""
    shape, stride, es = tuple(t.shape), tuple(t.stride()), t.element_size()
    for d in (i for i, n in enumerate(shape) if n == num_blocks):
        per_block = prod(shape[d + 1:])
        outer = prod(shape[:d])
        dense = per_block > 0 and _packed(shape[d + 1:], stride[d + 1:]) and stride[d] >= per_block
        if not dense or (outer > 1 and d != 1):
            continue
        layout = TensorLayout(base=t.data_ptr(), outer=outer, outer_stride=stride[0] * es if outer > 1 else 0,
                              block_stride=stride[d] * es, seg_bytes=per_block * es, num_blocks=num_blocks)
        if heads_dims is None:
            return layout
        tok_d, head_d = (x % len(shape) for x in heads_dims)
        head_bytes = es * prod(shape[max(tok_d, head_d) + 1:])
        return layout.with_heads(shape[head_d], stride[head_d] * es, shape[tok_d], stride[tok_d] * es, head_bytes)
    raise ValueError(f"no contiguous num_blocks={num_blocks} dimension in shape {shape} stride {stride}")


def find_heads_dims(shape: tuple, num_blocks: int, kv_heads: int, block_size: int,
                    layout: Optional[str] = None) -> Optional[Tuple[int, int]]:
    """(token dim, head dim) among the dims between the block dim and the
    last one, matched by size.  When the head count equals the block size
    the layout name decides: ``LBHNC`` puts heads first, ``LBNHC`` tokens."""
    if num_blocks not in shape or not kv_heads:
        return None
    between = list(range(list(shape).index(num_blocks) + 1, len(shape) - 1))
    head_d = [d for d in between if shape[d] == kv_heads]
    tok_d = [d for d in between if shape[d] == block_size]
    if not head_d or not tok_d:
        return None
    if kv_heads != block_size:
        return tok_d[0], head_d[0]
    if len(between) < 2:
        return None
    name = (layout or "").upper()
    heads_first = "H" in name and "N" in name and name.index("H") < name.index("N")
    a, b = between[0], between[1]
    return (b, a) if heads_first else (a, b)


def block_runs(local: Sequence[int], remote: Sequence[int]) -> List[Tuple[int, int, int]]:
    """(local_start, remote_start, count) runs where both lists advance by one."""
    if len(local) != len(remote):
        raise ValueError(f"block lists differ in length: {len(local)} vs {len(remote)}")
    # within a run, block - position is constant on both sides
    keyed = ((lb - i, rb - i, lb, rb) for i, (lb, rb) in enumerate(zip(local, remote)))
    runs = []
    for _, grp in itertools.groupby(keyed, key=lambda x: (x[0], x[1])):
        grp = list(grp)
        runs.append((grp[0][2], grp[0][3], len(grp)))
    return runs


def _pairs_checked(local_layouts, remote_layouts) -> List[Tuple[TensorLayout, TensorLayout]]:
    if len(local_layouts) != len(remote_layouts):
        raise ValueError(f"peer has {len(remote_layouts)} KV tensors, we have {len(local_layouts)}")
    return list(zip(local_layouts, remote_layouts))


def read_ops(local_layouts: Sequence[TensorLayout], remote_layouts: Sequence[TensorLayout],
             local_blocks: Sequence[int], remote_blocks: Sequence[int]) -> List[Op]:
    """Reads that copy the peer's ``remote_blocks`` into our ``local_blocks``."""
    pairs = _pairs_checked(local_layouts, remote_layouts)
    runs = block_runs(local_blocks, remote_blocks)
    ops: List[Op] = []
    for mine, theirs in pairs:
        if (mine.seg_bytes, mine.outer) != (theirs.seg_bytes, theirs.outer):
            raise ValueError(f"KV layout mismatch between instances (segment {mine.seg_bytes} vs "
                             f"{theirs.seg_bytes} bytes, {mine.outer} vs {theirs.outer} segments per block)")
        packed = mine.block_stride == mine.seg_bytes and theirs.block_stride == theirs.seg_bytes
        for o in range(mine.outer):
            for l0, r0, n in runs:
                if packed:
                    ops.append((mine.segment(o, l0), theirs.segment(o, r0), n * mine.seg_bytes))
                    continue
                ops += [(mine.segment(o, l0 + i), theirs.segment(o, r0 + i), mine.seg_bytes) for i in range(n)]
    return ops


def register_spans(layouts: Iterable[TensorLayout]) -> List[Tuple[int, int]]:
    """The memory spans to register: each layout's span, overlapping ones merged."""
    merged: List[List[int]] = []
    for start, length in sorted(lo.span for lo in layouts):
        end = start + length
        if merged and start < merged[-1][1]:
            merged[-1][1] = max(merged[-1][1], end)
        else:
            merged.append([start, end])
    return [(s, e - s) for s, e in merged]


@dataclass(frozen=True)
class TPSource:
    """A remote TP rank this local rank reads: ``nheads`` heads from remote
    head ``remote_head0`` to local head ``local_head0`` (both relative to
    their rank's shard); ``readers`` local ranks read that remote rank and
    the lowest of them (``releaser``) releases its hold."""

    remote_rank: int
    nheads: int
    local_head0: int
    remote_head0: int
    releaser: bool
    readers: int


def _shard(rank: int, per_rank: int) -> Tuple[int, int]:
    return rank * per_rank, (rank + 1) * per_rank


def tp_plan(local_rank: int, local_tp: int, remote_tp: int, total_heads: int) -> List[TPSource]:
    """What local rank ``local_rank`` reads when KV heads are sharded in
    contiguous equal ranges (rank r of a TP-t instance holds heads
    ``[r*H/t, (r+1)*H/t)``)."""
    for tp in (local_tp, remote_tp):
        if tp < 1 or total_heads % tp:
            raise ValueError(f"{total_heads} KV heads cannot be sharded over TP {tp} "
                             "(replicated KV heads are not supported)")
    if not 0 <= local_rank < local_tp:
        raise ValueError(f"rank {local_rank} outside TP {local_tp}")
    per_local, per_remote = total_heads // local_tp, total_heads // remote_tp
    lo, hi = _shard(local_rank, per_local)
    plan = []
    for p in range(remote_tp):
        r_lo, r_hi = _shard(p, per_remote)
        a, b = max(lo, r_lo), min(hi, r_hi)
        if a >= b:
            continue
        readers = range(r_lo // per_local, (r_hi - 1) // per_local + 1)   # local ranks overlapping shard p
        plan.append(TPSource(p, b - a, a - lo, a - r_lo, local_rank == readers[0], len(readers)))
    return plan


def _head_pieces(mine: TensorLayout, theirs: TensorLayout, my_h0: int, their_h0: int,
                 nheads: int) -> List[Op]:
    """(dst offset, src offset, bytes) inside one block segment for the head range."""
    if mine.head_major and theirs.head_major:       # one contiguous slab of heads
        return [(my_h0 * mine.head_stride, their_h0 * theirs.head_stride, nheads * mine.head_stride)]
    if mine.token_major and theirs.token_major:     # per token, the heads are adjacent
        return [(t * mine.token_stride + my_h0 * mine.head_bytes,
                 t * theirs.token_stride + their_h0 * theirs.head_bytes, nheads * mine.head_bytes)
                for t in range(mine.tokens)]
    return [((my_h0 + h) * mine.head_stride + t * mine.token_stride,
             (their_h0 + h) * theirs.head_stride + t * theirs.token_stride, mine.head_bytes)
            for h in range(nheads) for t in range(mine.tokens)]


def _coalesce(ops: Iterable[Op]) -> List[Op]:
    out: List[Op] = []
    for dst, src, n in ops:
        if out and out[-1][0] + out[-1][2] == dst and out[-1][1] + out[-1][2] == src:
            d0, s0, n0 = out[-1]
            out[-1] = (d0, s0, n0 + n)
        else:
            out.append((dst, src, n))
    return out


def head_read_ops(local_layouts: Sequence[TensorLayout], remote_layouts: Sequence[TensorLayout],
                  local_blocks: Sequence[int], remote_blocks: Sequence[int], local_head0: int,
                  remote_head0: int, nheads: int) -> List[Op]:
    """Reads copying remote heads ``[remote_head0, +nheads)`` of the peer's
    blocks into local heads ``[local_head0, +nheads)`` of ours; adjacent reads
    are merged."""
    pairs = _pairs_checked(local_layouts, remote_layouts)
    runs = block_runs(local_blocks, remote_blocks)

    def expand() -> Iterator[Op]:
        for mine, theirs in pairs:
            if not (mine.heads and theirs.heads):
                raise ValueError("KV head geometry unknown: cannot re-layout heads")
            if (mine.tokens, mine.head_bytes, mine.outer) != (theirs.tokens, theirs.head_bytes, theirs.outer):
                raise ValueError("KV layout mismatch between instances (block tokens / head bytes / segments)")
            if local_head0 + nheads > mine.heads or remote_head0 + nheads > theirs.heads:
                raise ValueError(f"head range outside the shard ({local_head0}+{nheads} of {mine.heads} local, "
                                 f"{remote_head0}+{nheads} of {theirs.heads} remote)")
            pieces = _head_pieces(mine, theirs, local_head0, remote_head0, nheads)
            for o in range(mine.outer):
                for l0, r0, n in runs:
                    for i in range(n):
                        dst, src = mine.segment(o, l0 + i), theirs.segment(o, r0 + i)
                        for d_off, s_off, length in pieces:
                            yield dst + d_off, src + s_off, length
    return _coalesce(expand())


def cx_cache_layouts(kv) -> List[TensorLayout]:
    """Layouts of a connex_b200 paged cache ``[L, 2, blocks, Hkv, BS, D]``: one
    per layer with K and V as the two segments, heads major (HND)."""
    L, _, nb, H, BS, D = kv.shape
    es = kv.element_size()
    st = [s * es for s in kv.stride()]
    return [TensorLayout(base=kv.data_ptr() + l * st[0], outer=2, outer_stride=st[1], block_stride=st[2],
                         seg_bytes=H * BS * D * es, num_blocks=nb).with_heads(H, st[3], BS, st[4], D * es)
            for l in range(L)]

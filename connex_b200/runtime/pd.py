"""Prefill -> decode disaggregation on B200: layer-by-layer paged-KV push.

The reference pulls a request's KV only after its whole prefill finished
(``connex/adapters/vllm/pd_connector.py:420-428``: the per-layer hooks are
no-ops; ``connex/pd/transfer.py:397-462`` issues one-sided reads).  Here the
prefill instance pushes instead, one kernel per layer:

* right after layer l's K/V land in the prefill cache (RoPE + cache-write
  kernel), an event is recorded on the compute stream and the push stream
  launches ``kv_push_layer`` for every (src block, dst block) pair of the
  batch -- so the transfer of layer l overlaps the compute of layers l+1..;
* the kernel stores straight into the decode instance's cache through its
  NVLink peer mapping (CUDA IPC) -- no staging, no host involvement -- and
  every CTA releases +1 on a u32 ready counter in the decode GPU's memory;
* the decode stream acquire-waits (bounded, status word on timeout) for the
  counter to reach the value the prefill side announced, then decodes.

The same kernel also runs on the *decode* GPU (:class:`LayerwiseKVPuller`):
the prefill stream then only publishes a per-layer ready counter in the
decode GPU's memory (:class:`LayerReadySignal`, one release store per
layer), and the decode stream acquire-waits for layer l and gathers layer
l's blocks from the prefill GPU's cache over NVLink into its own block
table.  The bytes and the overlap with the remaining prefill layers are the
same; the copy then uses the decode GPU's SMs, which sit idle while a
request is in prefill, instead of competing with the prefill's kernels.

Hold / acquire / release leases of :mod:`connex.pd.transfer` stay on the
host, so a decode instance that dies can still re-pull (the KV remains held
on the prefill side until released).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from connex_b200 import ops
from connex_b200.utils.nvtx import nvtx_range
from connex_b200.models.llama import LlamaModel, PagedKVCache, slot_mapping


@dataclass
class KVDestination:
    """Where a prefill instance writes KV: a decode cache (local or peer-mapped)."""

    base: int              # address of cache[0, 0] (layer 0, K)
    layer_stride: int      # bytes between layers
    kv_stride: int         # bytes between K and V of a layer
    heads: int             # KV heads per block in the destination cache
    num_blocks: int
    ready_addr: int        # u32 ready counter in the decode GPU's memory
    head_offset: int = 0   # first destination head written by this source

    @classmethod
    def of_cache(cls, cache: PagedKVCache, ready: torch.Tensor, base: Optional[int] = None,
                 ready_addr: Optional[int] = None) -> "KVDestination":
        return cls(base=base if base is not None else cache.kv.data_ptr(),
                   layer_stride=cache.layer_stride_bytes, kv_stride=cache.kv_stride_bytes,
                   heads=cache.cfg.kv_heads, num_blocks=cache.num_blocks,
                   ready_addr=ready_addr if ready_addr is not None else ready.data_ptr())

    def k(self, layer: int) -> int:
        return self.base + layer * self.layer_stride

    def v(self, layer: int) -> int:
        return self.base + layer * self.layer_stride + self.kv_stride


class LayerwiseKVPusher:
    """Launches one ``kv_push_layer`` per layer on a side stream, in step with
    the prefill's per-layer hook; counts the CTAs the decode side must see."""

    def __init__(self, src: PagedKVCache, max_ctas: int = 0, priority: int = -1, threads: int = 128):
        self.src = src
        # High priority: push CTAs take SM slots ahead of the queued prefill
        # CTAs.  The prefill's GEMM and attention kernels are persistent (one
        # CTA per SM, most of its shared memory); the attention kernel leaves
        # exactly the registers of one 128-thread push CTA free on each SM, so
        # the push runs beside them with one such CTA per SM (max_ctas 0: the
        # SM count) instead of waiting for a kernel to end.
        self.stream = torch.cuda.Stream(device=src.kv.device, priority=priority)
        self.status = ops.new_status(src.kv.device)
        self.max_ctas = max_ctas or torch.cuda.get_device_properties(src.kv.device).multi_processor_count
        self.threads = threads
        self._pairs: Optional[torch.Tensor] = None
        self._dst: Optional[KVDestination] = None
        self.launched = 0
        self.bytes = 0
        self.timing = False
        self._ev: List[tuple] = []
        self._span: Optional[torch.Tensor] = None

    def begin(self, pairs: torch.Tensor, dst: KVDestination, n_heads: Optional[int] = None,
              src_h0: int = 0, timing: bool = False) -> None:
        self._pairs, self._dst = pairs, dst
        self._nh = n_heads if n_heads is not None else self.src.cfg.kv_heads
        self._sh0 = src_h0
        self.launched = 0
        self.bytes = 0
        self.timing = timing
        self._ev = []
        if timing:
            L = self.src.cfg.layers
            if self._span is None or self._span.shape[0] < L:
                self._span = torch.empty(L, 2, dtype=torch.int64, device=self.src.kv.device)
            self._span[:, 0] = -1          # u64 max: the kernels lower it to their first start
            self._span[:, 1] = 0

    def hook(self, layer: int) -> None:
        """Called on the host right after layer ``layer``'s KV write was enqueued."""
        cur = torch.cuda.current_stream(self.src.kv.device)
        ev = torch.cuda.Event()
        ev.record(cur)
        self.stream.wait_event(ev)
        d, c = self._dst, self.src
        with torch.cuda.stream(self.stream), nvtx_range(f"kv push {layer}"):
            if self.timing:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
            n = ops.kv_push_layer(c.k(layer).data_ptr(), c.v(layer).data_ptr(), d.k(layer), d.v(layer),
                                  self._pairs, src_heads=c.cfg.kv_heads, dst_heads=d.heads,
                                  src_h0=self._sh0, dst_h0=d.head_offset, n_heads=self._nh,
                                  chunk_bytes=c.head_slice_bytes, src_blocks=c.num_blocks,
                                  dst_blocks=d.num_blocks, ready=d.ready_addr, max_ctas=self.max_ctas,
                                  status=self.status,
                                  span=self._span[layer].data_ptr() if self.timing else 0, threads=self.threads)
            if self.timing:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record(self.stream)
                self._ev.append((e0, e1))
        self.launched += n
        self.bytes += self._pairs.shape[0] * 2 * self._nh * c.head_slice_bytes

    def push_ms(self) -> float:
        """Summed time of this batch's push launches from their stream's point
        of view (CUDA events around each launch; needs timing=True, synced)."""
        return sum(a.elapsed_time(b) for a, b in self._ev)

    def kernel_ms(self) -> float:
        """Summed execution windows of this batch's push kernels as the
        kernels themselves saw them (first CTA start to last CTA end)."""
        if not self._ev:
            return 0.0
        sp = self._span[:len(self._ev)].cpu()
        return float((sp[:, 1] - sp[:, 0]).clamp(min=0).sum()) * 1e-6

    def span_events(self):
        return (self._ev[0][0], self._ev[-1][1]) if self._ev else (None, None)

    def join(self) -> None:
        torch.cuda.current_stream(self.src.kv.device).wait_stream(self.stream)


class LayerReadySignal:
    """Prefill side of the pull design: right after layer l's KV write the
    compute stream stores ``base + l + 1`` (release, system scope) into the
    decode GPU's layer counter (a peer-mapped u32).  Use ``hook`` as the
    prefill's ``layer_hook``."""

    def __init__(self, counter_addr: int, device, layers: int):
        self.addr, self.layers = counter_addr, layers
        self.like = torch.empty(1, device=device)
        self.base = 0

    def begin(self) -> int:
        """Start a batch; returns the counter base the decode side waits from."""
        return self.base

    def hook(self, layer: int) -> None:
        ops.write_flag(self.addr, self.base + layer + 1, self.like)

    def end(self) -> None:
        self.base += self.layers


class LayerwiseKVPuller:
    """Decode side of the pull design: for every layer, a bounded
    acquire-wait on the layer counter, then one ``kv_push_layer`` launch that
    gathers the layer's (src block, dst block) pairs from the prefill GPU's
    peer-mapped cache into the local cache.  Everything is enqueued up front
    on the decode stream; the waits hold the pulls back until the prefill
    publishes each layer."""

    def __init__(self, dst: PagedKVCache, max_ctas: int = 0, timeout_s: float = 30.0):
        self.dst = dst
        self.max_ctas = max_ctas
        self.timeout_s = timeout_s
        self.status = ops.new_status(dst.kv.device)
        self.bytes = 0
        self._ev: List[tuple] = []
        self._span: Optional[torch.Tensor] = None

    def pull(self, src_base: int, src_layer_stride: int, src_kv_stride: int, src_heads: int, src_blocks: int,
             pairs: torch.Tensor, counter_addr: int, base: int, timing: bool = False, src_h0: int = 0,
             dst_h0: int = 0, n_heads: Optional[int] = None) -> None:
        """Enqueue the whole batch's pulls on the current stream."""
        c = self.dst
        L = c.cfg.layers
        nh = n_heads if n_heads is not None else c.cfg.kv_heads
        self._ev = []
        self.bytes = 0
        if timing:
            if self._span is None or self._span.shape[0] < L:
                self._span = torch.empty(L, 2, dtype=torch.int64, device=c.kv.device)
            self._span[:, 0] = -1
            self._span[:, 1] = 0
        stream = torch.cuda.current_stream(c.kv.device)
        for layer in range(L):
            ops.wait_flag(counter_addr, base + layer + 1, self.status, timeout_s=self.timeout_s)
            with nvtx_range(f"kv pull {layer}"):
                if timing:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                sk = src_base + layer * src_layer_stride
                ops.kv_push_layer(sk, sk + src_kv_stride, c.k(layer).data_ptr(), c.v(layer).data_ptr(), pairs,
                                  src_heads=src_heads, dst_heads=c.cfg.kv_heads, src_h0=src_h0, dst_h0=dst_h0,
                                  n_heads=nh, chunk_bytes=c.head_slice_bytes, src_blocks=src_blocks,
                                  dst_blocks=c.num_blocks, max_ctas=self.max_ctas, status=self.status,
                                  span=self._span[layer].data_ptr() if timing else 0)
                if timing:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(stream)
                    self._ev.append((e0, e1))
            self.bytes += pairs.shape[0] * 2 * nh * c.head_slice_bytes

    def pull_ms(self) -> float:
        """Summed device time of the pull launches (CUDA events; waits excluded)."""
        return sum(a.elapsed_time(b) for a, b in self._ev)

    def kernel_ms(self) -> float:
        if not self._ev:
            return 0.0
        sp = self._span[:len(self._ev)].cpu()
        return float((sp[:, 1] - sp[:, 0]).clamp(min=0).sum()) * 1e-6


@dataclass
class PrefillBatch:
    """A packed prefill batch with its device-side metadata."""

    seq_lens: List[int]
    ids: torch.Tensor
    positions: torch.Tensor
    slots: torch.Tensor
    last_rows: torch.Tensor
    tile_info: torch.Tensor
    src_blocks: List[List[int]]

    @property
    def tokens(self) -> int:
        return sum(self.seq_lens)


def build_prefill_batch(cache: PagedKVCache, prompts: Sequence[Sequence[int]], device,
                        ids: Optional[torch.Tensor] = None,
                        blocks: Optional[Sequence[Sequence[int]]] = None) -> PrefillBatch:
    """Allocate source blocks (or use ``blocks``, allocated earlier) and build
    positions / slots / tile metadata.  ``ids`` may be given already on the
    device (e.g. copied from pinned memory)."""
    bs = cache.cfg.block_size
    seq_lens = [len(p) for p in prompts]
    given = list(blocks) if blocks is not None else None
    blocks, pos, slots, rows = [], [], [], []
    r = 0
    for i, n in enumerate(seq_lens):
        b = list(given[i]) if given is not None else cache.allocate(cache.blocks_needed(n))
        blocks.append(b)
        pos.extend(range(n))
        slots.extend(slot_mapping(b, 0, n, bs))
        r += n
        rows.append(r - 1)
    if ids is None:
        flat = [t for p in prompts for t in p]
        ids = torch.tensor(flat, dtype=torch.int32).pin_memory().to(device, non_blocking=True)
    return PrefillBatch(seq_lens=seq_lens, ids=ids,
                        positions=torch.tensor(pos, dtype=torch.int32).pin_memory().to(device, non_blocking=True),
                        slots=torch.tensor(slots, dtype=torch.int64).pin_memory().to(device, non_blocking=True),
                        last_rows=torch.tensor(rows, dtype=torch.int32).pin_memory().to(device, non_blocking=True),
                        tile_info=ops.prefill_tile_info(seq_lens, device), src_blocks=blocks)


def block_pairs(src_blocks: Sequence[Sequence[int]], dst_blocks: Sequence[Sequence[int]], device) -> torch.Tensor:
    flat = [(s, d) for sb, db in zip(src_blocks, dst_blocks) for s, d in zip(sb, db)]
    return torch.tensor(flat, dtype=torch.int32).pin_memory().to(device, non_blocking=True)


class DecodeBatch:
    """Device metadata of one decode step for sequences whose KV is in `cache`."""

    def __init__(self, cache: PagedKVCache, blocks: Sequence[Sequence[int]], ctx_lens: Sequence[int], device):
        bs = cache.cfg.block_size
        self.B = len(blocks)
        maxb = max(len(b) for b in blocks)
        self.block_tables = torch.tensor([list(b) + [0] * (maxb - len(b)) for b in blocks],
                                         dtype=torch.int32).to(device, non_blocking=True)
        # position of the new token = current context length (before append)
        self.positions = torch.tensor(list(ctx_lens), dtype=torch.int32).to(device, non_blocking=True)
        self.slots = torch.tensor([slot_mapping(b, n, 1, bs)[0] for b, n in zip(blocks, ctx_lens)],
                                  dtype=torch.int64).to(device, non_blocking=True)
        self.ctx_lens = (self.positions + 1)
        self.max_ctx = max(ctx_lens) + 1
        self.rows = torch.arange(self.B, dtype=torch.int32, device=device)


def decode_step(model: LlamaModel, batch: DecodeBatch, ids: torch.Tensor, workspace: torch.Tensor) -> torch.Tensor:
    return model.decode(ids, batch.positions, batch.slots, batch.block_tables, batch.ctx_lens, batch.max_ctx,
                        workspace, batch.rows)

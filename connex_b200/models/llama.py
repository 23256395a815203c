"""Llama-3-architecture decoder on connex_b200's own sm_100a kernels.

Weights are random-init N(0, 0.02) from a seed (there is no checkpoint to
load); the architecture is Llama-3-8B's by default (32 layers, hidden 4096,
32 q heads / 8 kv heads of 128, FFN 14336, vocab 128256, RoPE theta 5e5).

Storage layout, chosen for the kernels rather than for checkpoint parity:

* ``wqkv``  [(Hq + 2 Hkv) * 128, H]  -- q, k, v projections stacked (fused QKV GEMM)
* ``w13``   [2 F, H]                 -- gate/up interleaved per 256-row tile so the
                                        GEMM epilogue emits SiLU(gate) * up directly
* ``wo``, ``w2``                     -- consumed with the residual-add epilogue
* paged KV cache [L, 2, blocks, Hkv, 16, 128]: one head of one block is a
  contiguous 4 KB slice, the unit the PD push kernel moves.

The forward passes launch only this package's kernels (tcgen05 GEMM,
RMSNorm, RoPE + cache write, attention, argmax); a per-layer hook lets the
PD path launch the KV push of layer l while layers l+1.. still compute.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import torch

from connex_b200 import ops
from connex_b200.utils import nvtx


@dataclass(frozen=True)
class LlamaConfig:
    vocab_size: int = 128256
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    rope_theta: float = 500000.0
    eps: float = 1e-5
    max_pos: int = 8192 + 512
    block_size: int = 16
    rope_scaling: Optional[tuple] = None     # (factor, low_freq_factor, high_freq_factor, original_max_pos)

    @classmethod
    def llama3_8b(cls) -> "LlamaConfig":
        return cls()

    @classmethod
    def llama31_8b(cls) -> "LlamaConfig":
        """Llama-3.1-8B: the 8B geometry with 128k positions and Llama 3.1 RoPE scaling."""
        return cls(max_pos=131072, rope_scaling=(8.0, 1.0, 4.0, 8192))

    @classmethod
    def tiny(cls, layers: int = 2) -> "LlamaConfig":
        """A small config with the same head geometry (for tests / smoke)."""
        return cls(vocab_size=1024, hidden=512, layers=layers, heads=8, kv_heads=2, ffn=1024,
                   max_pos=2048)

    @property
    def qkv_dim(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def kv_bytes_per_token(self) -> int:
        return 2 * self.layers * self.kv_heads * self.head_dim * 2

    def num_params(self) -> int:
        per_layer = self.qkv_dim * self.hidden + self.hidden * self.heads * self.head_dim \
            + 3 * self.ffn * self.hidden + 2 * self.hidden
        return self.layers * per_layer + 2 * self.vocab_size * self.hidden + self.hidden


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor
    wo: torch.Tensor
    mlp_norm: torch.Tensor
    w13: torch.Tensor
    w2: torch.Tensor


@dataclass
class LlamaWeights:
    cfg: LlamaConfig
    embed: torch.Tensor
    layers: List[LayerWeights]
    final_norm: torch.Tensor
    lm_head: torch.Tensor

    @classmethod
    def random(cls, cfg: LlamaConfig, device, seed: int = 0, std: float = 0.02) -> "LlamaWeights":
        g = torch.Generator(device=device)
        g.manual_seed(seed)

        def rnd(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=device)
            t.normal_(0.0, std, generator=g)
            return t

        def ones(n):
            return torch.ones(n, dtype=torch.bfloat16, device=device)

        layers = []
        for _ in range(cfg.layers):
            gate, up = rnd(cfg.ffn, cfg.hidden), rnd(cfg.ffn, cfg.hidden)
            layers.append(LayerWeights(
                attn_norm=ones(cfg.hidden),
                wqkv=rnd(cfg.qkv_dim, cfg.hidden),
                wo=rnd(cfg.hidden, cfg.heads * cfg.head_dim),
                mlp_norm=ones(cfg.hidden),
                w13=ops.interleave_gate_up(gate, up),
                w2=rnd(cfg.hidden, cfg.ffn),
            ))
            del gate, up
        return cls(cfg=cfg, embed=rnd(cfg.vocab_size, cfg.hidden), layers=layers,
                   final_norm=ones(cfg.hidden), lm_head=rnd(cfg.vocab_size, cfg.hidden))

    @staticmethod
    def layout(cfg: LlamaConfig):
        """``(name, shape)`` of every engine tensor, in :meth:`named_tensors` order."""
        yield "model.embed_tokens.weight", (cfg.vocab_size, cfg.hidden)
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            yield p + "input_layernorm.weight", (cfg.hidden,)
            yield p + "self_attn.qkv_proj.weight", (cfg.qkv_dim, cfg.hidden)
            yield p + "self_attn.o_proj.weight", (cfg.hidden, cfg.heads * cfg.head_dim)
            yield p + "post_attention_layernorm.weight", (cfg.hidden,)
            yield p + "mlp.gate_up_proj.weight", (2 * cfg.ffn, cfg.hidden)
            yield p + "mlp.down_proj.weight", (cfg.hidden, cfg.ffn)
        yield "model.norm.weight", (cfg.hidden,)
        yield "lm_head.weight", (cfg.vocab_size, cfg.hidden)

    @classmethod
    def from_arena(cls, cfg: LlamaConfig, arena: torch.Tensor, manifest) -> "LlamaWeights":
        """Weights as views into one uint8 arena laid out by ``manifest``
        (a ``connex.rl.weights.WeightManifest`` of :meth:`layout`)."""
        t = {e.name: arena[e.offset:e.offset + e.nbytes].view(torch.bfloat16).view(e.shape)
             for e in manifest.entries}
        layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            layers.append(LayerWeights(attn_norm=t[p + "input_layernorm.weight"],
                                       wqkv=t[p + "self_attn.qkv_proj.weight"], wo=t[p + "self_attn.o_proj.weight"],
                                       mlp_norm=t[p + "post_attention_layernorm.weight"],
                                       w13=t[p + "mlp.gate_up_proj.weight"], w2=t[p + "mlp.down_proj.weight"]))
        return cls(cfg=cfg, embed=t["model.embed_tokens.weight"], layers=layers, final_norm=t["model.norm.weight"],
                   lm_head=t["lm_head.weight"])

    def named_tensors(self):
        """(name, tensor) in HF-style naming with fused qkv / gate_up tensors."""
        yield "model.embed_tokens.weight", self.embed
        for i, lw in enumerate(self.layers):
            p = f"model.layers.{i}."
            yield p + "input_layernorm.weight", lw.attn_norm
            yield p + "self_attn.qkv_proj.weight", lw.wqkv
            yield p + "self_attn.o_proj.weight", lw.wo
            yield p + "post_attention_layernorm.weight", lw.mlp_norm
            yield p + "mlp.gate_up_proj.weight", lw.w13
            yield p + "mlp.down_proj.weight", lw.w2
        yield "model.norm.weight", self.final_norm
        yield "lm_head.weight", self.lm_head


def trainer_layout(cfg: LlamaConfig):
    """``(name, shape)`` of the unfused HF checkpoint tensors a trainer holds."""
    yield "model.embed_tokens.weight", (cfg.vocab_size, cfg.hidden)
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        yield p + "input_layernorm.weight", (cfg.hidden,)
        yield p + "self_attn.q_proj.weight", (cfg.heads * cfg.head_dim, cfg.hidden)
        yield p + "self_attn.k_proj.weight", (cfg.kv_heads * cfg.head_dim, cfg.hidden)
        yield p + "self_attn.v_proj.weight", (cfg.kv_heads * cfg.head_dim, cfg.hidden)
        yield p + "self_attn.o_proj.weight", (cfg.hidden, cfg.heads * cfg.head_dim)
        yield p + "post_attention_layernorm.weight", (cfg.hidden,)
        yield p + "mlp.gate_proj.weight", (cfg.ffn, cfg.hidden)
        yield p + "mlp.up_proj.weight", (cfg.ffn, cfg.hidden)
        yield p + "mlp.down_proj.weight", (cfg.hidden, cfg.ffn)
    yield "model.norm.weight", (cfg.hidden,)
    yield "lm_head.weight", (cfg.vocab_size, cfg.hidden)


def random_trainer_weights(cfg: LlamaConfig, device, dtype=torch.float32, seed: int = 0, std: float = 0.02):
    """Random unfused HF-named weights (e.g. a trainer's fp32 master copy)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for name, shape in trainer_layout(cfg):
        t = torch.empty(shape, dtype=dtype, device=device)
        if "norm" in name:
            t.uniform_(0.5, 1.5, generator=g)
        else:
            t.normal_(0.0, std, generator=g)
        out[name] = t
    return out


class PagedKVCache:
    """Paged KV cache [L, 2, blocks, Hkv, BS, D] with a free-block allocator."""

    def __init__(self, cfg: LlamaConfig, num_blocks: int, device, dtype=torch.bfloat16,
                 storage: Optional[torch.Tensor] = None):
        self.cfg = cfg
        self.num_blocks = num_blocks
        shape = (cfg.layers, 2, num_blocks, cfg.kv_heads, cfg.block_size, cfg.head_dim)
        self.kv = storage.view(shape) if storage is not None else torch.empty(shape, dtype=dtype, device=device)
        self._free = list(range(num_blocks - 1, -1, -1))

    def k(self, layer: int) -> torch.Tensor:
        return self.kv[layer, 0]

    def v(self, layer: int) -> torch.Tensor:
        return self.kv[layer, 1]

    @property
    def head_slice_bytes(self) -> int:
        return self.cfg.block_size * self.cfg.head_dim * self.kv.element_size()

    @property
    def layer_stride_bytes(self) -> int:
        return self.kv.stride(0) * self.kv.element_size()

    @property
    def kv_stride_bytes(self) -> int:
        return self.kv.stride(1) * self.kv.element_size()

    def blocks_needed(self, n_tokens: int) -> int:
        return (n_tokens + self.cfg.block_size - 1) // self.cfg.block_size

    def allocate(self, n_blocks: int) -> List[int]:
        if n_blocks > len(self._free):
            raise MemoryError(f"KV cache exhausted: need {n_blocks}, have {len(self._free)}")
        return [self._free.pop() for _ in range(n_blocks)]

    def free(self, blocks: Sequence[int]) -> None:
        self._free.extend(reversed(list(blocks)))

    @property
    def free_blocks(self) -> int:
        return len(self._free)


def slot_mapping(block_ids: Sequence[int], start: int, n: int, block_size: int) -> List[int]:
    return [block_ids[(start + i) // block_size] * block_size + (start + i) % block_size for i in range(n)]


LayerHook = Callable[[int], None]


class LlamaModel:
    """Forward passes of the Llama decoder over a :class:`PagedKVCache`."""

    def __init__(self, weights: LlamaWeights, cache: PagedKVCache, max_tokens: int, max_batch: int = 256,
                 tp=None):
        """``tp``: a :class:`connex_b200.parallel.tp.TPGroup` when ``weights``
        are one rank's shard (``shard_llama``); the residual stream is then
        all-reduced after the o- and down-projections."""
        self.w = weights
        self.tp = tp
        self.cfg = weights.cfg
        self.cache = cache
        cfg = self.cfg
        dev = weights.embed.device
        self.device = dev
        self.cos_sin = ops.rope_cos_sin(cfg.max_pos, cfg.head_dim, cfg.rope_theta, dev, cfg.rope_scaling)
        self.status = ops.new_status(dev)
        self.max_tokens = max_tokens
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.empty(max_tokens, cfg.hidden, **bf)
        self.h = torch.empty(max_tokens, cfg.hidden, **bf)
        self.qkv = torch.empty(max_tokens, cfg.qkv_dim, **bf)
        self.attn = torch.empty(max_tokens, cfg.heads * cfg.head_dim, **bf)
        self.mid = torch.empty(max_tokens, cfg.ffn, **bf)
        self.last = torch.empty(max_batch, cfg.hidden, **bf)
        self.logits = torch.empty(max_batch, cfg.vocab_size, **bf)
        self.next_ids = torch.empty(max_batch, dtype=torch.int32, device=dev)
        self.max_batch = max_batch

    # ------------------------------------------------------------ layers
    def _residual_gemm(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor) -> None:
        """x += a @ w^T; under tensor parallelism summed over the group: rank 0
        adds its partial to x in the epilogue, the others store theirs into
        x, and an all-reduce of x adds them up."""
        tp = self.tp
        if tp is None or tp.world == 1:
            ops.gemm(a, w, x, residual=x, status=self.status)
            return
        ops.gemm(a, w, x, residual=x if tp.rank == 0 else None, status=self.status)
        tp.all_reduce(x)

    def _layer_tail(self, l: int, T: int):
        cfg, lw = self.cfg, self.w.layers[l]
        x, h = self.x[:T], self.h[:T]
        self._residual_gemm(self.attn[:T], lw.wo, x)
        ops.rmsnorm(x, lw.mlp_norm, cfg.eps, out=h)
        ops.gemm(h, lw.w13, self.mid[:T], silu_mul=True, status=self.status)
        self._residual_gemm(self.mid[:T], lw.w2, x)
        nw = self.w.layers[l + 1].attn_norm if l + 1 < cfg.layers else self.w.final_norm
        ops.rmsnorm(x, nw, cfg.eps, out=h)

    def _head(self, rows: torch.Tensor, B: int) -> torch.Tensor:
        last = self.last[:B]
        ops.gather_rows(self.h, rows, last)
        logits = self.logits[:B]
        ops.gemm(last, self.w.lm_head, logits, status=self.status)
        return ops.argmax(logits, self.next_ids[:B])

    def prefill(self, ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                seq_lens: Sequence[int], last_rows: torch.Tensor, tile_info: torch.Tensor,
                layer_hook: Optional[LayerHook] = None, hook_after_attention: bool = False) -> torch.Tensor:
        """Prefill a packed batch; returns the greedy next token of each sequence.

        ``layer_hook(l)`` runs (on the host, in stream order) right after layer
        l's K/V are in the paged cache: the PD path launches its push there.
        With ``hook_after_attention`` it runs after layer l's attention has
        been enqueued instead (the push then overlaps the layer's GEMMs rather
        than its attention kernel)."""
        cfg, T = self.cfg, ids.numel()
        assert T <= self.max_tokens
        nvtx.push(f"prefill T={T}")
        ops.embedding(ids, self.w.embed, self.x[:T], status=self.status)
        ops.rmsnorm(self.x[:T], self.w.layers[0].attn_norm, cfg.eps, out=self.h[:T])
        for l, lw in enumerate(self.w.layers):
            nvtx.push(f"layer {l}")
            qkv = self.qkv[:T]
            ops.gemm(self.h[:T], lw.wqkv, qkv, status=self.status)
            ops.rope_cache(qkv, positions, self.cos_sin, cfg.heads, cfg.kv_heads, slots,
                           self.cache.k(l), self.cache.v(l), status=self.status)
            if layer_hook is not None and not hook_after_attention:
                layer_hook(l)
            ops.prefill_attention(qkv, tile_info, cfg.heads, cfg.kv_heads, out=self.attn[:T])
            if layer_hook is not None and hook_after_attention:
                layer_hook(l)
            self._layer_tail(l, T)
            nvtx.pop()
        out = self._head(last_rows, len(seq_lens))
        nvtx.pop()
        return out

    def decode(self, ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
               block_tables: torch.Tensor, ctx_lens: torch.Tensor, max_ctx: int,
               workspace: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
        """One decode step for B sequences (ctx_lens include the new token)."""
        cfg, B = self.cfg, ids.numel()
        nvtx.push(f"decode B={B}")
        ops.embedding(ids, self.w.embed, self.x[:B], status=self.status)
        ops.rmsnorm(self.x[:B], self.w.layers[0].attn_norm, cfg.eps, out=self.h[:B])
        for l, lw in enumerate(self.w.layers):
            qkv = self.qkv[:B]
            ops.gemm(self.h[:B], lw.wqkv, qkv, status=self.status)
            ops.rope_cache(qkv, positions, self.cos_sin, cfg.heads, cfg.kv_heads, slots,
                           self.cache.k(l), self.cache.v(l), status=self.status)
            ops.decode_attention(qkv, self.cache.k(l), self.cache.v(l), block_tables, ctx_lens,
                                 cfg.heads, max_ctx, workspace, out=self.attn[:B])
            self._layer_tail(l, B)
        out = self._head(rows, B)
        nvtx.pop()
        return out


# ------------------------------------------------------------- oracle
def reference_forward(weights: LlamaWeights, seqs: Sequence[Sequence[int]]) -> List[torch.Tensor]:
    """fp32 PyTorch forward (no cache) returning last-position logits per sequence."""
    from connex_b200.ops import reference as R
    cfg = weights.cfg
    cos_sin = ops.rope_cos_sin(cfg.max_pos, cfg.head_dim, cfg.rope_theta, weights.embed.device,
                               cfg.rope_scaling)
    outs = []
    for seq in seqs:
        ids = torch.tensor(seq, device=weights.embed.device)
        n = len(seq)
        pos = torch.arange(n, device=ids.device)
        x = weights.embed[ids].float()
        for lw in weights.layers:
            h = R.rmsnorm(x, lw.attn_norm, cfg.eps)
            qkv = h @ lw.wqkv.float().t()
            q = qkv[:, :cfg.heads * 128].view(n, cfg.heads, 128)
            k = qkv[:, cfg.heads * 128:(cfg.heads + cfg.kv_heads) * 128].view(n, cfg.kv_heads, 128)
            v = qkv[:, (cfg.heads + cfg.kv_heads) * 128:].view(n, cfg.kv_heads, 128)
            q, k = R.rope(q, pos, cos_sin), R.rope(k, pos, cos_sin)
            a = R.causal_attention(q, k, v, [n]).reshape(n, -1)
            x = x + a @ lw.wo.float().t()
            h = R.rmsnorm(x, lw.mlp_norm, cfg.eps)
            x = x + R.silu_mul_gemm(h, lw.w13) @ lw.w2.float().t()
        h = R.rmsnorm(x[-1:], weights.final_norm, cfg.eps)
        outs.append((h @ weights.lm_head.float().t())[0])
    return outs

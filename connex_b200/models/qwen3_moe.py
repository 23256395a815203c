"""Qwen3-MoE-style decoder (Qwen3-30B-A3B geometry by default) served with
data-parallel attention and expert-parallel MoE layers on sm_100a.

Per layer: RMSNorm -> fused QKV GEMM -> per-head q/k RMSNorm + RoPE + paged
KV write (one kernel) -> paged decode / varlen prefill attention -> output
projection with the residual add in the GEMM epilogue -> RMSNorm -> MoE
(:class:`connex_b200.parallel.ep.EPMoE`: dispatch over NVLink peer memory,
tcgen05 grouped expert GEMMs, combine) -> residual add fused into the next
layer's RMSNorm.  Each rank runs attention for its own requests; the
experts of a layer are spread over the ranks' slots (``S`` per rank) and
found through the placement's logical -> physical map, so a migrated expert
serves from its new slot at the next step.

Routing follows the benchmark workload: router logits ~ N(0, 1) plus a
seeded Zipf(1.2) popularity bias (:func:`zipf_router`), top-k, weights
renormalised.  Expert ``e`` of layer ``l`` has weights drawn from the seed
``(seed, l, e)``, wherever it is placed, so a migrated copy can be checked
against a freshly drawn one.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from connex_b200 import ops


@dataclass(frozen=True)
class Qwen3MoeConfig:
    vocab_size: int = 151936
    hidden: int = 2048
    layers: int = 48
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    moe_ffn: int = 768
    rope_theta: float = 1000000.0
    eps: float = 1e-6
    max_pos: int = 8192
    block_size: int = 16

    @classmethod
    def qwen3_30b_a3b(cls) -> "Qwen3MoeConfig":
        return cls()

    @classmethod
    def tiny(cls, layers: int = 2) -> "Qwen3MoeConfig":
        return cls(vocab_size=1024, hidden=512, layers=layers, heads=8, kv_heads=2, experts=16, top_k=4,
                   moe_ffn=256, max_pos=2048)

    @property
    def qkv_dim(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def expert_bytes_per_layer(self) -> int:
        return 3 * self.moe_ffn * self.hidden * 2


def expert_weights(cfg: Qwen3MoeConfig, layer: int, expert: int, device, seed: int = 0, std: float = 0.02):
    """(w13 [2F, H] gate/up interleaved, w2 [H, F]) of one expert, bf16."""
    g = torch.Generator(device=device)
    g.manual_seed(((seed * 1009 + layer) * 100003 + expert) & 0x7FFFFFFFFFFF)
    F, H = cfg.moe_ffn, cfg.hidden
    gate = torch.empty(F, H, dtype=torch.bfloat16, device=device).normal_(0, std, generator=g)
    up = torch.empty(F, H, dtype=torch.bfloat16, device=device).normal_(0, std, generator=g)
    w2 = torch.empty(H, F, dtype=torch.bfloat16, device=device).normal_(0, std, generator=g)
    return ops.interleave_gate_up(gate, up), w2


def zipf_router(T: int, cfg: Qwen3MoeConfig, gen: torch.Generator, bias: torch.Tensor):
    """Top-k routing of T tokens from N(0,1) logits + a Zipf popularity bias."""
    logits = torch.randn(T, cfg.experts, generator=gen, device=bias.device) + bias
    w, idx = torch.topk(torch.softmax(logits, -1), cfg.top_k, dim=-1)
    return idx.to(torch.int32).contiguous(), (w / w.sum(-1, keepdim=True)).float().contiguous()


def zipf_bias(cfg: Qwen3MoeConfig, seed: int, device, skew: float = 1.2) -> torch.Tensor:
    ranks = np.random.default_rng(seed).permutation(cfg.experts) + 1
    return torch.tensor(-skew * np.log(ranks), dtype=torch.float32, device=device)


@dataclass
class AttnLayer:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    wo: torch.Tensor
    mlp_norm: torch.Tensor


class Qwen3MoeRank:
    """One EP rank: replicated attention weights, its expert slots, its KV cache."""

    def __init__(self, cfg: Qwen3MoeConfig, rank: int, slots_per_rank: int, placement: List[List[int]], device,
                 num_blocks: int, max_tokens: int, seed: int = 0):
        """``placement[l][p]``: logical expert in physical slot ``p`` of layer
        ``l`` (-1 = empty); this rank holds slots ``[rank*S, (rank+1)*S)``."""
        self.cfg, self.rank, self.S, self.device = cfg, rank, slots_per_rank, torch.device(device)
        dev = self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 7 + 11)

        def rnd(*shape):
            return torch.empty(*shape, dtype=torch.bfloat16, device=dev).normal_(0, 0.02, generator=g)

        def ones(n):
            return torch.ones(n, dtype=torch.bfloat16, device=dev)
        self.embed = rnd(cfg.vocab_size, cfg.hidden)
        self.lm_head = rnd(cfg.vocab_size, cfg.hidden)
        self.final_norm = ones(cfg.hidden)
        self.attn: List[AttnLayer] = [AttnLayer(ones(cfg.hidden), rnd(cfg.qkv_dim, cfg.hidden), ones(cfg.head_dim),
                                                ones(cfg.head_dim), rnd(cfg.hidden, cfg.heads * cfg.head_dim),
                                                ones(cfg.hidden)) for _ in range(cfg.layers)]
        S, F, H = slots_per_rank, cfg.moe_ffn, cfg.hidden
        self.w13 = torch.zeros(cfg.layers, S, 2 * F, H, dtype=torch.bfloat16, device=dev)
        self.w2 = torch.zeros(cfg.layers, S, H, F, dtype=torch.bfloat16, device=dev)
        for l in range(cfg.layers):
            for j in range(S):
                e = placement[l][rank * S + j]
                if e >= 0:
                    a, b = expert_weights(cfg, l, e, dev, seed)
                    self.w13[l, j].copy_(a)
                    self.w2[l, j].copy_(b)
        from connex_b200.models.llama import LlamaConfig, PagedKVCache
        kv_cfg = LlamaConfig(vocab_size=cfg.vocab_size, hidden=cfg.hidden, layers=cfg.layers, heads=cfg.heads,
                             kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, block_size=cfg.block_size)
        self.cache = PagedKVCache(kv_cfg, num_blocks, dev)
        self.cos_sin = ops.rope_cos_sin(cfg.max_pos, cfg.head_dim, cfg.rope_theta, dev)
        self.status = ops.new_status(dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.max_tokens = max_tokens
        self.x = torch.empty(max_tokens, H, **bf)
        self.h = torch.empty(max_tokens, H, **bf)
        self.qkv = torch.empty(max_tokens, cfg.qkv_dim, **bf)
        self.att = torch.empty(max_tokens, cfg.heads * cfg.head_dim, **bf)
        self.moe_out = torch.empty(max_tokens, H, **bf)
        self.logits = torch.empty(max_tokens, cfg.vocab_size, **bf)
        self.next_ids = torch.empty(max_tokens, dtype=torch.int32, device=dev)
        self.moe = None          # EPMoE, attached by the serving loop

    def expert_slot_views(self, layer: int, local_slot: int):
        return self.w13[layer, local_slot], self.w2[layer, local_slot]

    def decode(self, ids, positions, slots, block_tables, ctx_lens, max_ctx, workspace, routing, l2p, l2p_cnt):
        """One decode step of this rank's batch; ``routing[l] = (topk_idx, topk_w)``."""
        cfg, T = self.cfg, ids.numel()
        x, h = self.x[:T], self.h[:T]
        ops.embedding(ids, self.embed, x, status=self.status)
        ops.rmsnorm(x, self.attn[0].attn_norm, cfg.eps, out=h)
        for l, a in enumerate(self.attn):
            qkv = self.qkv[:T]
            ops.gemm(h, a.wqkv, qkv, status=self.status)
            ops.rope_cache(qkv, positions, self.cos_sin, cfg.heads, cfg.kv_heads, slots, self.cache.k(l),
                           self.cache.v(l), status=self.status, q_norm=a.q_norm, k_norm=a.k_norm, eps=cfg.eps)
            ops.decode_attention(qkv, self.cache.k(l), self.cache.v(l), block_tables, ctx_lens, cfg.heads, max_ctx,
                                 workspace, out=self.att[:T])
            ops.gemm(self.att[:T], a.wo, x, residual=x, status=self.status)
            ops.rmsnorm(x, a.mlp_norm, cfg.eps, out=h)
            self.moe.w13 = self.w13[l].reshape(-1, cfg.hidden)
            self.moe.w2 = self.w2[l].reshape(-1, cfg.moe_ffn)
            idx, w = routing[l]
            out = self.moe.forward(h, idx, w, l2p[l], l2p_cnt[l], self.moe_out[:T])
            nw = self.attn[l + 1].attn_norm if l + 1 < cfg.layers else self.final_norm
            ops.rmsnorm(out, nw, cfg.eps, out=h, residual=x)      # x += moe; h = norm(x)
        logits = self.logits[:T]
        ops.gemm(h, self.lm_head, logits, status=self.status)
        return ops.argmax(logits, self.next_ids[:T])

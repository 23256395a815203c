"""Tensor parallelism for the Llama runtime (Megatron-style column / row
splits with one all-reduce after each row-parallel projection).

Per layer, rank r of W holds:

* ``wqkv``: the q rows of query heads ``[r*Hq/W, (r+1)*Hq/W)`` and the k and v
  rows of KV heads ``[r*Hkv/W, (r+1)*Hkv/W)`` (GQA groups stay whole), so
  attention and the paged KV cache are local to the rank (Hkv/W heads);
* ``wo``: the matching input columns (row-parallel);
* ``w13``: FFN rows ``[r*F/W, (r+1)*F/W)`` of gate and of up, interleaved
  again in the SiLU-mul GEMM's 128-row blocks (column-parallel);
* ``w2``: the matching input columns (row-parallel).

Embedding, norms and the LM head are replicated.  After ``wo`` and after
``w2`` the ranks' partial sums are added by an all-reduce of the residual
stream (``LlamaModel._residual_gemm`` with ``tp=TPGroup``): rank 0 runs the
GEMM with the residual epilogue (x + its partial), the others store their
partial into x, and the all-reduce (sum) leaves x + sum of partials on every
rank -- no extra buffer or add kernel.

The all-reduce is NCCL's (NVLS inside an NVSwitch box when NCCL selects it)
on the compute stream, so decode CUDA graphs capture it.  Reference: TP in
the reference is vLLM's / SGLang's (``connex/pp/group.py`` and
``connex/pd/group.py`` handle the membership side, which this framework
keeps in the same files).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from connex_b200 import ops
from connex_b200.models.llama import LayerWeights, LlamaConfig, LlamaWeights

HEAD_DIM = 128


@dataclass
class TPGroup:
    """A tensor-parallel group: ``rank`` of ``world`` in process group ``pg``."""
    rank: int
    world: int
    pg: Optional[object] = None

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.pg)


def tp_config(cfg: LlamaConfig, world: int) -> LlamaConfig:
    """The per-rank geometry (heads, KV heads and FFN width divided by ``world``)."""
    if cfg.heads % world or cfg.kv_heads % world:
        raise ValueError(f"{cfg.heads} query / {cfg.kv_heads} KV heads do not split over {world} ranks")
    half = ops.GATE_UP_TILE // 2
    if cfg.ffn % (world * half):
        raise ValueError(f"FFN width {cfg.ffn} does not split over {world} ranks in {half}-row blocks")
    return LlamaConfig(**{**cfg.__dict__, "heads": cfg.heads // world, "kv_heads": cfg.kv_heads // world,
                          "ffn": cfg.ffn // world})


def shard_layer(lw: LayerWeights, cfg: LlamaConfig, rank: int, world: int) -> LayerWeights:
    hq, hkv = cfg.heads // world, cfg.kv_heads // world
    q0 = cfg.heads * HEAD_DIM
    qs = lw.wqkv[rank * hq * HEAD_DIM:(rank + 1) * hq * HEAD_DIM]
    ks = lw.wqkv[q0 + rank * hkv * HEAD_DIM:q0 + (rank + 1) * hkv * HEAD_DIM]
    v0 = q0 + cfg.kv_heads * HEAD_DIM
    vs = lw.wqkv[v0 + rank * hkv * HEAD_DIM:v0 + (rank + 1) * hkv * HEAD_DIM]
    f = cfg.ffn // world
    gate, up = ops.deinterleave_gate_up(lw.w13)
    return LayerWeights(
        attn_norm=lw.attn_norm,
        wqkv=torch.cat([qs, ks, vs], 0).contiguous(),
        wo=lw.wo[:, rank * hq * HEAD_DIM:(rank + 1) * hq * HEAD_DIM].contiguous(),
        mlp_norm=lw.mlp_norm,
        w13=ops.interleave_gate_up(gate[rank * f:(rank + 1) * f], up[rank * f:(rank + 1) * f]),
        w2=lw.w2[:, rank * f:(rank + 1) * f].contiguous())


def shard_llama(w: LlamaWeights, rank: int, world: int) -> LlamaWeights:
    """Rank ``rank``'s weights (per-rank config; replicated embedding, norms and head)."""
    return LlamaWeights(cfg=tp_config(w.cfg, world), embed=w.embed,
                        layers=[shard_layer(lw, w.cfg, rank, world) for lw in w.layers],
                        final_norm=w.final_norm, lm_head=w.lm_head)


def reference_tp_forward(weights: LlamaWeights, seqs, world: int):
    """fp32 oracle of the sharded computation: every rank's partial sums
    added exactly (an ideal all-reduce); last-position logits per sequence."""
    from connex_b200.ops import reference as R
    cfg = weights.cfg
    shards = [shard_llama(weights, r, world) for r in range(world)]
    cos_sin = ops.rope_cos_sin(cfg.max_pos, cfg.head_dim, cfg.rope_theta, weights.embed.device, cfg.rope_scaling)
    outs = []
    for seq in seqs:
        ids = torch.tensor(seq, device=weights.embed.device)
        n = len(seq)
        pos = torch.arange(n, device=ids.device)
        x = weights.embed[ids].float()
        for li in range(cfg.layers):
            h = R.rmsnorm(x, weights.layers[li].attn_norm, cfg.eps)
            part = torch.zeros_like(x)
            for sh in shards:
                lw, c = sh.layers[li], sh.cfg
                qkv = h @ lw.wqkv.float().t()
                q = qkv[:, :c.heads * HEAD_DIM].view(n, c.heads, HEAD_DIM)
                k = qkv[:, c.heads * HEAD_DIM:(c.heads + c.kv_heads) * HEAD_DIM].view(n, c.kv_heads, HEAD_DIM)
                v = qkv[:, (c.heads + c.kv_heads) * HEAD_DIM:].view(n, c.kv_heads, HEAD_DIM)
                q, k = R.rope(q, pos, cos_sin), R.rope(k, pos, cos_sin)
                a = R.causal_attention(q, k, v, [n]).reshape(n, -1)
                part += a @ lw.wo.float().t()
            x = x + part
            h = R.rmsnorm(x, weights.layers[li].mlp_norm, cfg.eps)
            part = torch.zeros_like(x)
            for sh in shards:
                lw = sh.layers[li]
                part += R.silu_mul_gemm(h, lw.w13) @ lw.w2.float().t()
            x = x + part
        h = R.rmsnorm(x[-1:], weights.final_norm, cfg.eps)
        outs.append((h @ weights.lm_head.float().t())[0])
    return outs

"""Plain PyTorch fp32 re-statements of every kernel in :mod:`connex_b200.ops`.

These are the numerics oracles of the test-suite (and of ``smoke()``); no
production code path calls them.  Each takes the same arguments as its
kernel counterpart and returns fp32 results computed from the bf16 inputs.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def gemm(a, b, residual=None):
    out = a.float() @ b.float().t()
    if residual is not None:
        out = out + residual.float()
    return out


def silu_mul_gemm(a, w_interleaved, tile=256):
    from connex_b200.ops import deinterleave_gate_up  # noqa: WPS433 (pure torch helper)
    g, u = deinterleave_gate_up(w_interleaved, tile)
    return F.silu(a.float() @ g.float().t()) * (a.float() @ u.float().t())


def rmsnorm(x, w, eps, residual=None):
    xf = x.float()
    if residual is not None:
        xf = (xf + residual.float()).to(torch.bfloat16).float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return xf * torch.rsqrt(var + eps) * w.float()


def rope(x, positions, cos_sin):
    """x: [T, H, 128] -> rotated (rotate-half convention)."""
    d = x.shape[-1]
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, : d // 2], cs[:, None, d // 2:]
    x1, x2 = x[..., : d // 2].float(), x[..., d // 2:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def causal_attention(q, k, v, seq_lens, scale=None):
    """q [T, Hq, D], k/v [T, Hkv, D] packed by sequence -> [T, Hq, D] fp32."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty(T, Hq, D, dtype=torch.float32, device=q.device)
    s = 0
    for n in seq_lens:
        qs = q[s:s + n].float().transpose(0, 1)  # [Hq, n, D]
        ks = k[s:s + n].float().transpose(0, 1).repeat_interleave(Hq // Hkv, 0)
        vs = v[s:s + n].float().transpose(0, 1).repeat_interleave(Hq // Hkv, 0)
        att = (qs @ ks.transpose(1, 2)) * scale
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1)
        att = att.masked_fill(mask, float("-inf")).softmax(-1)
        out[s:s + n] = (att @ vs).transpose(0, 1)
        s += n
    return out


def paged_decode_attention(q, k_cache, v_cache, block_tables, ctx_lens, scale=None):
    """q [B, Hq, D]; caches [blocks, Hkv, BS, D] -> [B, Hq, D] fp32."""
    B, Hq, D = q.shape
    Hkv, BS = k_cache.shape[1], k_cache.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        n = int(ctx_lens[b])
        nb = (n + BS - 1) // BS
        blocks = block_tables[b, :nb].long()
        k = k_cache[blocks].float().permute(1, 0, 2, 3).reshape(Hkv, nb * BS, D)[:, :n]
        v = v_cache[blocks].float().permute(1, 0, 2, 3).reshape(Hkv, nb * BS, D)[:, :n]
        k = k.repeat_interleave(Hq // Hkv, 0)
        v = v.repeat_interleave(Hq // Hkv, 0)
        att = (q[b].float()[:, None, :] @ k.transpose(1, 2)) * scale  # [Hq, 1, n]
        out[b] = (att.softmax(-1) @ v)[:, 0]
    return out


def paged_prefill_attention(q, k_cache, v_cache, block_tables, ctx, n_new, scale=None):
    """Chunks that continue cached sequences: q [T, Hq, D] packed by sequence
    (``n_new[i]`` rows each); K/V of positions [0, ctx[i] + n_new[i]) from the
    caches [blocks, Hkv, BS, D] through ``block_tables``; query j of sequence
    i sits at position ctx[i] + j -> [T, Hq, D] fp32."""
    T, Hq, D = q.shape
    Hkv, BS = k_cache.shape[1], k_cache.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty(T, Hq, D, dtype=torch.float32, device=q.device)
    s = 0
    for b, (c, n) in enumerate(zip(ctx, n_new)):
        tot = c + n
        nb = (tot + BS - 1) // BS
        blocks = block_tables[b, :nb].long()
        k = k_cache[blocks].float().permute(1, 0, 2, 3).reshape(Hkv, nb * BS, D)[:, :tot]
        v = v_cache[blocks].float().permute(1, 0, 2, 3).reshape(Hkv, nb * BS, D)[:, :tot]
        k = k.repeat_interleave(Hq // Hkv, 0)
        v = v.repeat_interleave(Hq // Hkv, 0)
        qs = q[s:s + n].float().transpose(0, 1)                        # [Hq, n, D]
        att = (qs @ k.transpose(1, 2)) * scale                         # [Hq, n, tot]
        keys = torch.arange(tot, device=q.device)[None, :]
        pos = (c + torch.arange(n, device=q.device))[:, None]
        att = att.masked_fill(keys > pos, float("-inf")).softmax(-1)
        out[s:s + n] = (att @ v).transpose(0, 1)
        s += n
    return out


def kv_push(src_k, src_v, dst_k, dst_v, pairs, src_h0=0, dst_h0=0, n_heads=None):
    """In-place reference of kv_push_layer on plain tensors."""
    nh = n_heads if n_heads is not None else src_k.shape[1]
    for sb, db in pairs.tolist():
        dst_k[db, dst_h0:dst_h0 + nh] = src_k[sb, src_h0:src_h0 + nh]
        dst_v[db, dst_h0:dst_h0 + nh] = src_v[sb, src_h0:src_h0 + nh]

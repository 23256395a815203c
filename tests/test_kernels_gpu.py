"""Numerics of every sm_100a kernel against its fp32 PyTorch re-statement."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    return torch.device("cuda", 0)


def _rnd(*shape, dev, std=1.0, seed=0):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)


def _close(out, ref, rtol=2e-2, atol=2e-2):
    out = out.float()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= atol + rtol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (300, 768, 512), (1, 256, 128),
                                   (17, 1024, 4096), (1000, 4096, 1024), (64, 6144, 4096)])
def test_gemm(dev, M, N, K):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    a, b = _rnd(M, K, dev=dev, seed=1), _rnd(N, K, dev=dev, seed=2)
    st = ops.new_status(dev)
    out = ops.gemm(a, b, status=st)
    torch.cuda.synchronize()
    ops.check_status(st, "gemm")
    _close(out, R.gemm(a, b))


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_tile_widths(dev, bn):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    a, b = _rnd(513, 1024, dev=dev, seed=3), _rnd(2048, 1024, dev=dev, seed=4)
    out = ops.gemm(a, b, bn=bn)
    _close(out, R.gemm(a, b))


def test_gemm_residual_inplace(dev):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    a, b = _rnd(200, 512, dev=dev, seed=5), _rnd(768, 512, dev=dev, seed=6)
    x = _rnd(200, 768, dev=dev, seed=7)
    ref = R.gemm(a, b, residual=x)
    ops.gemm(a, b, x, residual=x)
    _close(x, ref)


def test_gemm_silu_mul(dev):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    a = _rnd(333, 512, dev=dev, seed=8)
    gate, up = _rnd(1024, 512, dev=dev, seed=9, std=0.1), _rnd(1024, 512, dev=dev, seed=10, std=0.1)
    w = ops.interleave_gate_up(gate, up)
    out = ops.gemm(a, w, silu_mul=True)
    assert out.shape == (333, 1024)
    _close(out, R.silu_mul_gemm(a, w))


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
def test_gemm_skinny_rows(dev, M):
    """Decode-sized GEMMs (M <= 8) run the weight-streaming kernel: store,
    in-place residual on a strided output view and SiLU-mul epilogues vs the
    fp32 reference, one launch each, and a K that is not a multiple of 256."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    assert ops._C.gemm_splits(M, 4096, 4096, ops.EPI_STORE, 0) == 1
    for K in (4096, 1032):
        a, b = _rnd(M, K, dev=dev, seed=30 + M), _rnd(1544, K, dev=dev, seed=31)
        n0 = ops.launch_count()
        out = ops.gemm(a, b)
        assert ops.launch_count() == n0 + 1
        _close(out, R.gemm(a, b))
    a, b = _rnd(M, 4096, dev=dev, seed=32), _rnd(2048, 4096, dev=dev, seed=33)
    big = _rnd(M, 4096, dev=dev, seed=34)
    x = big[:, 1024:3072]                       # row stride 4096, 16-byte aligned
    ref = R.gemm(a, b, residual=x)
    ops.gemm(a, b, x, residual=x)
    _close(x, ref)
    gate, up = _rnd(1024, 4096, dev=dev, seed=35, std=0.1), _rnd(1024, 4096, dev=dev, seed=36, std=0.1)
    w = ops.interleave_gate_up(gate, up)
    _close(ops.gemm(a, w, silu_mul=True), R.silu_mul_gemm(a, w))


@pytest.mark.parametrize("M", [16, 64, 130])
def test_gemm_split_k(dev, M):
    """Small-M (decode) GEMMs split the K loop: plain, residual and SiLU-mul
    epilogues against the fp32 reference; the workspace is left zero."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    a, b = _rnd(M, 4096, dev=dev, seed=20), _rnd(1024, 4096, dev=dev, seed=21)
    assert ops._C.gemm_splits(M, 1024, 4096, ops.EPI_STORE, 0) > 1
    st = ops.new_status(dev)
    n0 = ops.launch_count()
    out = ops.gemm(a, b, status=st)
    assert ops.launch_count() == n0 + 2
    _close(out, R.gemm(a, b))
    x = _rnd(M, 1024, dev=dev, seed=22)
    ref = R.gemm(a, b, residual=x)
    ops.gemm(a, b, x, residual=x, splits=4)
    _close(x, ref)
    gate, up = _rnd(512, 4096, dev=dev, seed=23, std=0.1), _rnd(512, 4096, dev=dev, seed=24, std=0.1)
    w = ops.interleave_gate_up(gate, up)
    _close(ops.gemm(a, w, silu_mul=True, splits=8), R.silu_mul_gemm(a, w))
    torch.cuda.synchronize()
    ops.check_status(st, "gemm split-k")
    assert float(ops._SPLIT_WS[a.device].abs().max()) == 0.0


def test_rmsnorm(dev):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    for H in (512, 2048, 4096):
        x, w = _rnd(37, H, dev=dev, seed=11), _rnd(H, dev=dev, seed=12)
        _close(ops.rmsnorm(x, w, 1e-5), R.rmsnorm(x, w, 1e-5))
        res = _rnd(37, H, dev=dev, seed=13)
        ref = R.rmsnorm(x, w, 1e-5, residual=res)
        ref_res = (x.float() + res.float())
        out = ops.rmsnorm(x, w, 1e-5, residual=res)
        _close(out, ref)
        _close(res, ref_res)


def test_rope_cache(dev):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    Hq, Hkv, T, BS, NB = 8, 2, 40, 16, 10
    qkv = _rnd(T, (Hq + 2 * Hkv) * 128, dev=dev, seed=14)
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    cs = ops.rope_cos_sin(4096, 128, 500000.0, dev)
    slots = torch.randperm(NB * BS, device=dev)[:T].to(torch.int64)
    kc = torch.zeros(NB, Hkv, BS, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    orig = qkv.clone()
    ops.rope_cache(qkv, pos, cs, Hq, Hkv, slots, kc, vc)
    q = orig[:, :Hq * 128].view(T, Hq, 128)
    k = orig[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    v = orig[:, (Hq + Hkv) * 128:].view(T, Hkv, 128)
    _close(qkv[:, :Hq * 128].view(T, Hq, 128), R.rope(q, pos, cs))
    kr = R.rope(k, pos, cs)
    _close(qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128), kr)
    for t in range(T):
        s = int(slots[t])
        _close(kc[s // BS, :, s % BS], kr[t])
        assert torch.equal(vc[s // BS, :, s % BS], v[t])


def test_rope_cache_qk_norm(dev):
    """Per-head q/k RMSNorm (Qwen3) fused before the rotation."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    Hq, Hkv, T = 8, 2, 33
    qkv = _rnd(T, (Hq + 2 * Hkv) * 128, dev=dev, seed=31, std=0.5)
    pos = torch.randint(0, 2000, (T,), device=dev, dtype=torch.int32)
    cs = ops.rope_cos_sin(2048, 128, 1e6, dev)
    qn, kn = _rnd(128, dev=dev, seed=32) + 1, _rnd(128, dev=dev, seed=33) + 1
    orig = qkv.clone()
    ops.rope_cache(qkv, pos, cs, Hq, Hkv, q_norm=qn.bfloat16(), k_norm=kn.bfloat16(), eps=1e-6)

    def ref(x, w):
        n = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.bfloat16().float()
        return R.rope(n.bfloat16(), pos, cs)
    q = orig[:, :Hq * 128].view(T, Hq, 128)
    k = orig[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    _close(qkv[:, :Hq * 128].view(T, Hq, 128), ref(q, qn))
    _close(qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128), ref(k, kn))
    assert torch.equal(qkv[:, (Hq + Hkv) * 128:], orig[:, (Hq + Hkv) * 128:])


def test_embedding_argmax(dev):
    from connex_b200 import ops
    table = _rnd(1000, 256, dev=dev, seed=15)
    ids = torch.randint(0, 1000, (33,), device=dev, dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])
    logits = _rnd(5, 128256, dev=dev, seed=16)
    assert torch.equal(ops.argmax(logits).long(), logits.float().argmax(-1))


@pytest.mark.parametrize("lens", [[1], [128], [100, 37, 1], [513, 130, 7], [1100], [300, 256], [4096]])
@pytest.mark.parametrize("G", [4, 1])
@pytest.mark.parametrize("tile", [256, 128])
def test_prefill_attention(dev, lens, G, tile):
    """Both kernels (two 128-row Q tiles per CTA, or one) against the fp32
    reference: partial and empty second tiles, a 32-key-tile sequence."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    Hkv = 2
    Hq, T = Hkv * G, sum(lens)
    qkv = _rnd(T, (Hq + 2 * Hkv) * 128, dev=dev, seed=31)
    ti = ops.prefill_tile_info(lens, dev, tile_rows=tile)
    st = ops.new_status(dev)
    out = ops.prefill_attention(qkv, ti, Hq, Hkv, status=st, tile_rows=tile)
    torch.cuda.synchronize()
    ops.check_status(st, "prefill_attention")
    q = qkv[:, :Hq * 128].view(T, Hq, 128)
    k = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    v = qkv[:, (Hq + Hkv) * 128:].view(T, Hkv, 128)
    _close(out.view(T, Hq, 128), R.causal_attention(q, k, v, lens))


@pytest.mark.parametrize("split", [1, 2, 4])
@pytest.mark.parametrize("tile", [256, 128])
def test_prefill_attention_with_fma_pipe_exponentials(dev, split, tile):
    """Part of the softmax's 2^x on the FMA pipe (own cubic for 2^f): the
    output stays within the fp32 reference's tolerance."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    lens, Hkv, G = [513, 130, 7], 2, 4
    Hq, T = Hkv * G, sum(lens)
    qkv = _rnd(T, (Hq + 2 * Hkv) * 128, dev=dev, seed=41)
    ti = ops.prefill_tile_info(lens, dev, tile_rows=tile)
    try:
        ops._C.attention_exp_split(split)
        out = ops.prefill_attention(qkv, ti, Hq, Hkv, tile_rows=tile)
        torch.cuda.synchronize()
    finally:
        ops._C.attention_exp_split(0)
    q = qkv[:, :Hq * 128].view(T, Hq, 128)
    k = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    v = qkv[:, (Hq + Hkv) * 128:].view(T, Hkv, 128)
    _close(out.view(T, Hq, 128), R.causal_attention(q, k, v, lens))


@pytest.mark.parametrize("G", [4, 8])
def test_decode_attention(dev, G):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    Hkv, BS, NB = 2, 16, 640
    Hq = Hkv * G
    ctx = [1, 17, 600, 2000]
    B = len(ctx)
    kc, vc = _rnd(NB, Hkv, BS, 128, dev=dev, seed=18), _rnd(NB, Hkv, BS, 128, dev=dev, seed=19)
    maxb = (max(ctx) + BS - 1) // BS
    perm = torch.randperm(NB, device=dev).to(torch.int32)
    bt = perm[:B * maxb].view(B, maxb).contiguous()
    cl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    q = _rnd(B, Hq * 128 + 512, dev=dev, seed=20)  # extra columns: strided q rows
    ws = ops.decode_workspace(B, Hq, max(ctx), dev)
    out = ops.decode_attention(q, kc, vc, bt, cl, Hq, max(ctx), ws)
    ref = R.paged_decode_attention(q[:, :Hq * 128].view(B, Hq, 128), kc, vc, bt, cl)
    _close(out.view(B, Hq, 128), ref)
    # a workspace sized for a larger batch lets this small batch cut the context finer
    big = ops.decode_workspace(64, Hq, max(ctx), dev)
    assert ops._C.decode_attention_plan(B, Hq, Hkv, max(ctx), big.numel()) > \
        ops._C.decode_attention_plan(B, Hq, Hkv, max(ctx), ws.numel())
    out2 = ops.decode_attention(q, kc, vc, bt, cl, Hq, max(ctx), big)
    _close(out2.view(B, Hq, 128), ref)
    one = ops.decode_attention(q[3:], kc, vc, bt[3:], cl[3:], Hq, max(ctx), big)    # batch 1, 2000 tokens
    _close(one.view(1, Hq, 128), ref[3:])


@pytest.mark.parametrize("G", [1, 2])
def test_decode_attention_small_groups_and_unwritten_slots(dev, G):
    """GQA groups of 1 and 2, and cache slots past each sequence's end that
    hold NaN (never written): they must not reach the output."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    Hkv, BS, NB = 4, 16, 700
    Hq = Hkv * G
    ctx = [5, 16, 33, 1000, 2047]
    B = len(ctx)
    kc, vc = _rnd(NB, Hkv, BS, 128, dev=dev, seed=21), _rnd(NB, Hkv, BS, 128, dev=dev, seed=22)
    maxb = (max(ctx) + BS - 1) // BS
    perm = torch.randperm(NB, device=dev).to(torch.int32)
    bt = perm[:B * maxb].view(B, maxb).contiguous()
    for b, n in enumerate(ctx):                      # poison the tail of each last block
        if n % BS:
            last = int(bt[b, (n - 1) // BS])
            kc[last, :, n % BS:].view(torch.int16).fill_(-1)
            vc[last, :, n % BS:].view(torch.int16).fill_(-1)
    cl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    q = _rnd(B, Hq * 128, dev=dev, seed=23)
    ref = R.paged_decode_attention(q.reshape(B, Hq, 128), kc, vc, bt, cl)
    for ws in (ops.decode_workspace(B, Hq, max(ctx), dev), ops.decode_workspace(64, Hq, max(ctx), dev)):
        out = ops.decode_attention(q, kc, vc, bt, cl, Hq, max(ctx), ws)
        assert torch.isfinite(out.float()).all()
        _close(out.reshape(B, Hq, 128), ref)


def test_kv_push_local(dev):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    H, BS, NB = 8, 16, 64
    sk, sv = _rnd(NB, H, BS, 128, dev=dev, seed=21), _rnd(NB, H, BS, 128, dev=dev, seed=22)
    dk, dv = torch.zeros(2 * NB, H, BS, 128, dtype=torch.bfloat16, device=dev), \
        torch.zeros(2 * NB, H, BS, 128, dtype=torch.bfloat16, device=dev)
    pairs = torch.tensor([[i, 2 * i + 1] for i in range(0, NB, 3)], dtype=torch.int32, device=dev)
    flag = torch.zeros(4, dtype=torch.int32, device=dev)
    st = ops.new_status(dev)
    n = ops.kv_push_layer(sk.data_ptr(), sv.data_ptr(), dk.data_ptr(), dv.data_ptr(), pairs,
                          src_heads=H, dst_heads=H, chunk_bytes=BS * 128 * 2, src_blocks=NB,
                          dst_blocks=2 * NB, ready=flag.data_ptr(), status=st)
    ops.wait_flag(flag.data_ptr(), n, st, timeout_s=1.0)
    torch.cuda.synchronize()
    ops.check_status(st, "kv_push")
    assert int(flag[0]) == n
    rk, rv = torch.zeros_like(dk), torch.zeros_like(dv)
    R.kv_push(sk, sv, rk, rv, pairs.cpu())
    assert torch.equal(dk, rk) and torch.equal(dv, rv)


def test_kv_push_head_relayout(dev):
    """Prefill TP1 (8 heads) -> two decode ranks of TP2 (4 heads each)."""
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    BS, NB = 16, 8
    sk, sv = _rnd(NB, 8, BS, 128, dev=dev, seed=23), _rnd(NB, 8, BS, 128, dev=dev, seed=24)
    pairs = torch.tensor([[i, NB - 1 - i] for i in range(NB)], dtype=torch.int32, device=dev)
    for rank in range(2):
        dk = torch.zeros(NB, 4, BS, 128, dtype=torch.bfloat16, device=dev)
        dv = torch.zeros_like(dk)
        ops.kv_push_layer(sk.data_ptr(), sv.data_ptr(), dk.data_ptr(), dv.data_ptr(), pairs,
                          src_heads=8, dst_heads=4, src_h0=4 * rank, dst_h0=0, n_heads=4,
                          chunk_bytes=BS * 256, src_blocks=NB, dst_blocks=NB)
        rk, rv = torch.zeros_like(dk), torch.zeros_like(dv)
        R.kv_push(sk, sv, rk, rv, pairs.cpu(), src_h0=4 * rank, n_heads=4)
        torch.cuda.synchronize()
        assert torch.equal(dk, rk) and torch.equal(dv, rv)


def test_copy_segments(dev):
    from connex_b200 import ops
    src = torch.arange(1 << 20, dtype=torch.int32, device=dev)
    dst = torch.zeros_like(src)
    segs = torch.tensor([[src.data_ptr() + 64, dst.data_ptr() + 4096, 65536],
                         [src.data_ptr() + (1 << 20), dst.data_ptr() + (1 << 19), 1 << 18]], dtype=torch.int64)
    ops.copy_segments(segs.to(dev), 65536 + (1 << 18))
    torch.cuda.synchronize()
    d8, s8 = dst.view(torch.uint8), src.view(torch.uint8)
    assert torch.equal(d8[4096:4096 + 65536], s8[64:64 + 65536])
    assert torch.equal(d8[1 << 19:(1 << 19) + (1 << 18)], s8[1 << 20:(1 << 20) + (1 << 18)])


def test_wait_flag_times_out_with_status(dev):
    """A flag nothing sets: the bounded wait gives up and reports, no hang."""
    from connex_b200 import ops
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    st = ops.new_status(dev)
    ops.wait_flag(flag.data_ptr(), 1, st, timeout_s=0.05)
    torch.cuda.synchronize()
    assert int(st.item()) == 1
    # the context stays usable
    st2 = ops.new_status(dev)
    ops.write_flag(flag.data_ptr(), 5, flag)
    ops.wait_flag(flag.data_ptr(), 5, st2, timeout_s=1.0)
    torch.cuda.synchronize()
    assert int(st2.item()) == 0

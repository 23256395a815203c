"""The allocation-free decode-attention entry point, called through its C symbol.

``cx_decode_attention_noalloc`` serves callers that cannot call cudaMalloc
(engines that reserved all device memory up front; C callers without a
caching allocator, for whom cudaMalloc/cudaFree could synchronize the
device).  It keeps its split-K scratch in a fixed device array inside the
library.  This file is collected last on purpose: it must pass both on its
own in a fresh process and after every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

ERR_TOO_LARGE, ERR_ARGS = -1, -3


def _lib():
    from connex_b200 import _C
    lib = ctypes.CDLL(_C.__file__)
    f = lib.cx_decode_attention_noalloc
    f.restype = ctypes.c_int
    P, I = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [P, I, P, P, P, I, P, P, I, I, I, I, I, I, ctypes.c_float, P]
    lib.cx_noalloc_error_string.restype = ctypes.c_char_p
    lib.cx_noalloc_error_string.argtypes = [I]
    lib.cx_decode_attention_noalloc_scratch_floats.restype = ctypes.c_size_t
    lib.cx_decode_attention_noalloc_scratch_floats.argtypes = [I, I, I]
    return lib


def _case(dev, seed, ctx, G, Hkv=2, BS=16):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    Hq = Hkv * G
    maxb = (max(ctx) + BS - 1) // BS
    NB = len(ctx) * maxb + 8
    kc = torch.randn(NB, Hkv, BS, 128, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(NB, Hkv, BS, 128, generator=g, device=dev).to(torch.bfloat16)
    bt = torch.randperm(NB, device=dev)[:len(ctx) * maxb].to(torch.int32).view(len(ctx), maxb).contiguous()
    cl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    q = torch.randn(len(ctx), Hq * 128 + 256, generator=g, device=dev).to(torch.bfloat16)
    return q, kc, vc, bt, cl, Hq, Hkv, BS


def _call(lib, q, kc, vc, bt, cl, Hq, Hkv, BS, out, max_ctx):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.cx_decode_attention_noalloc(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
                                           bt.shape[1], cl.data_ptr(), out.data_ptr(), out.stride(0), q.shape[0],
                                           Hq, Hkv, BS, max_ctx, 1.0 / 128 ** 0.5, stream)


def _check(lib, dev, seed, ctx, G, max_ctx=None):
    """One call of the allocation-free entry point against the allocating
    entry point and the fp32 oracle."""
    from connex_b200 import ops
    from connex_b200.ops.reference import paged_decode_attention
    q, kc, vc, bt, cl, Hq, Hkv, BS = _case(dev, seed, ctx, G)
    max_ctx = max_ctx or max(ctx)
    ws = ops.decode_workspace(len(ctx), Hq, max_ctx, dev)
    ref = ops.decode_attention(q, kc, vc, bt, cl, Hq, max_ctx, ws)
    out = torch.full((len(ctx), Hq * 128), float("nan"), dtype=torch.bfloat16, device=dev)
    rc = _call(lib, q, kc, vc, bt, cl, Hq, Hkv, BS, out, max_ctx)
    assert rc == 0, lib.cx_noalloc_error_string(rc).decode()
    torch.cuda.synchronize(dev)
    err = (out.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err <= 2e-2 + 2e-2 * scale, f"vs allocating path: max err {err} vs scale {scale}"
    oracle = paged_decode_attention(q[:, :Hq * 128].float().view(len(ctx), Hq, 128), kc.float(), vc.float(),
                                    bt.long(), cl.long())
    err32 = (out.float().view_as(oracle) - oracle).abs().max().item()
    assert err32 <= 2e-2 + 2e-2 * oracle.abs().max().item(), f"vs fp32 oracle: max err {err32}"


def test_noalloc_matches_allocating_entry_point_twice():
    dev = torch.device("cuda", 0)
    lib = _lib()
    # two calls in a row, different sizes: the second reuses the scratch the first left behind
    for seed, ctx, G in [(1, [5, 700, 3000, 1200], 4), (2, [2100, 33], 8)]:
        _check(lib, dev, seed, ctx, G)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_noalloc_every_gqa_group(G):
    lib = _lib()
    dev = torch.device("cuda", 0)
    _check(lib, dev, 10 + G, [1, 17, 900], G)                  # one sequence per split regime
    # every sequence shorter than max_ctx: each split holds fewer live keys than its length
    _check(lib, dev, 20 + G, [40, 300, 129], G, max_ctx=2048)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib()
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, cl, Hq, Hkv, BS = _case(dev, 3, [64, 64], 4)
    out = torch.empty(2, Hq * 128, dtype=torch.bfloat16, device=dev)
    huge_ctx = 1 << 22  # needs far more than the built-in scratch
    assert lib.cx_decode_attention_noalloc_scratch_floats(2, Hq, huge_ctx) > (1 << 20)
    rc = _call(lib, q, kc, vc, bt, cl, Hq, Hkv, BS, out, huge_ctx)
    assert rc == ERR_TOO_LARGE
    assert b"scratch" in lib.cx_noalloc_error_string(rc)


def test_noalloc_rejects_unsupported_head_layouts():
    lib = _lib()
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, cl, Hq, Hkv, BS = _case(dev, 4, [64, 64], 4)
    out = torch.empty(2, Hq * 128, dtype=torch.bfloat16, device=dev)
    assert _call(lib, q, kc, vc, bt, cl, 6, 4, BS, out, 64) == ERR_ARGS        # Hq not a multiple of Hkv
    assert _call(lib, q, kc, vc, bt, cl, 32, 2, BS, out, 64) == ERR_ARGS       # GQA group 16
    assert b"GQA" in lib.cx_noalloc_error_string(ERR_ARGS)


def test_noalloc_second_device_has_its_own_scratch():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs a second GPU")
    lib = _lib()
    _check(lib, torch.device("cuda", 0), 5, [300, 40], 4)
    with torch.cuda.device(1):
        _check(lib, torch.device("cuda", 1), 6, [1000, 7], 8)     # resolves device 1's copy of the array
    _check(lib, torch.device("cuda", 0), 7, [64], 2)

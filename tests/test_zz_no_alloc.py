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


def test_noalloc_matches_allocating_entry_point_twice():
    from connex_b200 import ops
    dev = torch.device("cuda", 0)
    lib = _lib()
    # two calls in a row, different sizes: the second reuses the scratch the first left behind
    for seed, ctx, G in [(1, [5, 700, 3000, 1200], 4), (2, [2100, 33], 8)]:
        q, kc, vc, bt, cl, Hq, Hkv, BS = _case(dev, seed, ctx, G)
        max_ctx = max(ctx)
        ws = ops.decode_workspace(len(ctx), Hq, max_ctx, dev)
        ref = ops.decode_attention(q, kc, vc, bt, cl, Hq, max_ctx, ws)
        out = torch.full((len(ctx), Hq * 128), float("nan"), dtype=torch.bfloat16, device=dev)
        rc = _call(lib, q, kc, vc, bt, cl, Hq, Hkv, BS, out, max_ctx)
        assert rc == 0, lib.cx_noalloc_error_string(rc).decode()
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        scale = ref.float().abs().max().item() + 1e-6
        assert err <= 2e-2 + 2e-2 * scale, f"max err {err} vs scale {scale}"


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib()
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, cl, Hq, Hkv, BS = _case(dev, 3, [64, 64], 4)
    out = torch.empty(2, Hq * 128, dtype=torch.bfloat16, device=dev)
    huge_ctx = 1 << 22  # needs far more than the built-in scratch
    assert lib.cx_decode_attention_noalloc_scratch_floats(2, Hq, huge_ctx) > (1 << 20)
    rc = _call(lib, q, kc, vc, bt, cl, Hq, Hkv, BS, out, huge_ctx)
    assert rc == -1
    assert b"scratch" in lib.cx_noalloc_error_string(rc)

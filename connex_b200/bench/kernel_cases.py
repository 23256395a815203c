"""Single-kernel cases for timing and profiling the sm_100a kernels.

``python -m connex_b200.bench.kernel_cases <case> [--iters K]`` runs one
kernel on a fixed case (inputs larger than the 126 MB L2 where the kernel is
memory-bound, a few GB on the device at most), times it with CUDA events
after warm-up and prints one JSON line with the achieved rate and its
fraction of the measured peaks in ``MEASURED_PEAKS.json`` (copy bandwidth,
cuBLAS bf16 burst throughput).  The same command line is what a profiler
capture of the case runs.

Cases: gemm (8192^3), gemm_qkv (T=8192 Llama-3-8B QKV), gemm_silu (T=8192
gate/up + SiLU-mul), attn (8 x 2048-token causal prefill, 32/8 heads),
attn_paged (the paged variant: 8 chunks of 2048 queries over 2048 cached tokens), decode_attn (64 x 4096-token paged decode), kv_push (one layer of a 64k-token
KV push, local), kv_push_nvlink (the same layer pushed from GPU 0 into GPU 1's
memory over NVLink, one process, peer access; ``--ctas`` sets the grid,
``--pull`` runs the kernel on GPU 1 reading GPU 0's memory instead, ``--ce``
times a copy-engine peer copy of the same bytes for comparison),
kv_push_beside (the push of one 8k-token layer alone or next to a running
GEMM / attention kernel, ``--co``, ``--ctas``), wsync (Llama-3-8B 2-layer slice, fp32 -> bf16 fused
re-layout), ep_gemm (grouped expert GEMM, 1 GPU).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from connex_b200 import ops

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _time(fn, iters: int, warmup: int = 3, device=None) -> float:
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters


def _status_check(status, what):
    """A timed case's kernels record timeouts and bad arguments in a status
    word; a case whose kernels gave up is an error, not a slow number."""
    return lambda: ops.check_status(status, what)


def case_gemm(dev, M=8192, N=8192, K=8192, silu=False):
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(N, K, device=dev).bfloat16()
    out = torch.empty(M, N // 2 if silu else N, dtype=torch.bfloat16, device=dev)
    st = ops.new_status(dev)
    return (lambda: ops.gemm(a, b, out, silu_mul=silu, status=st)), {"flops": 2 * M * N * K,
                                                                      "check": _status_check(st, "gemm")}


def case_attn(dev, n_seq=8, L=2048, hq=32, hkv=8, tile=None):
    T = n_seq * L
    qkv = (torch.randn(T, (hq + 2 * hkv) * 128, device=dev) * 0.5).bfloat16()
    ti = ops.prefill_tile_info([L] * n_seq, dev, tile_rows=tile)
    out = torch.empty(T, hq * 128, dtype=torch.bfloat16, device=dev)
    flops = n_seq * hq * 2 * 2 * 128 * L * L / 2   # causal: half of QK^T and PV
    st = ops.new_status(dev)
    return (lambda: ops.prefill_attention(qkv, ti, hq, hkv, out, status=st, tile_rows=tile)), {
        "flops": flops, "check": _status_check(st, "prefill attention")}


def case_attn_library(dev, backend="cudnn", n_seq=8, L=2048, hq=32, hkv=8):
    """The same causal prefill (8 x 2048, 32 q / 8 kv heads, d=128) through
    torch's scaled_dot_product_attention on one of its library backends
    (cuDNN or torch's flash-attention kernels): a reference point for the
    tcgen05 kernel above.  K/V are expanded to the query heads outside the
    timed region."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    q = (torch.randn(n_seq, hq, L, 128, device=dev) * 0.5).bfloat16()
    k = (torch.randn(n_seq, hkv, L, 128, device=dev) * 0.5).bfloat16().repeat_interleave(hq // hkv, dim=1)
    v = (torch.randn(n_seq, hkv, L, 128, device=dev) * 0.5).bfloat16().repeat_interleave(hq // hkv, dim=1)
    be = {"cudnn": SDPBackend.CUDNN_ATTENTION, "flash": SDPBackend.FLASH_ATTENTION}[backend]
    flops = n_seq * hq * 2 * 2 * 128 * L * L / 2

    def run():
        with sdpa_kernel(be):
            F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return run, {"flops": flops}


def case_attn_paged(dev, n_seq=8, ctx=2048, L=2048, hq=32, hkv=8, tile=None):
    """Chunked prefill: 8 chunks of 2048 queries continuing 2048 cached tokens
    each, K/V of the whole context read from the paged cache."""
    bs = 16
    T = n_seq * L
    per = (ctx + L) // bs
    nb = n_seq * per
    kc = (torch.randn(nb, hkv, bs, 128, device=dev) * 0.5).bfloat16()
    vc = (torch.randn(nb, hkv, bs, 128, device=dev) * 0.5).bfloat16()
    bt = torch.randperm(nb, device=dev).to(torch.int32).view(n_seq, per).contiguous()
    qkv = (torch.randn(T, (hq + 2 * hkv) * 128, device=dev) * 0.5).bfloat16()
    ti = ops.prefill_tile_info([L] * n_seq, dev, ctx=[ctx] * n_seq, tile_rows=tile)
    out = torch.empty(T, hq * 128, dtype=torch.bfloat16, device=dev)
    flops = n_seq * hq * 4 * 128 * (L * ctx + L * L / 2)
    st = ops.new_status(dev)
    return (lambda: ops.prefill_attention_paged(qkv, kc, vc, bt, ti, hq, hkv, out, status=st, tile_rows=tile)), {
        "flops": flops, "check": _status_check(st, "paged prefill attention")}


def case_decode_attn(dev, B=64, ctx=4096, hq=32, hkv=8):
    bs = 16
    nb = B * ctx // bs
    k = torch.randn(nb, hkv, bs, 128, device=dev).bfloat16()
    v = torch.randn(nb, hkv, bs, 128, device=dev).bfloat16()
    bt = torch.arange(nb, dtype=torch.int32, device=dev).view(B, ctx // bs)
    cl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, hq * 128, device=dev).bfloat16()
    ws = ops.decode_workspace(B, hq, ctx, dev)
    out = torch.empty(B, hq * 128, dtype=torch.bfloat16, device=dev)
    return (lambda: ops.decode_attention(q, k, v, bt, cl, hq, ctx, ws, out)), {"bytes": 2 * k.numel() * 2}


def case_kv_push(dev, tokens=65536, hkv=8):
    bs = 16
    nb = tokens // bs
    src = torch.randn(2, nb, hkv, bs, 128, device=dev).bfloat16()
    dst = torch.empty_like(src)
    pairs = torch.stack([torch.arange(nb), torch.randperm(nb)], 1).int().to(dev)
    chunk = bs * 128 * 2

    def run():
        ops.kv_push_layer(src[0].data_ptr(), src[1].data_ptr(), dst[0].data_ptr(), dst[1].data_ptr(), pairs,
                          src_heads=hkv, dst_heads=hkv, chunk_bytes=chunk, src_blocks=nb, dst_blocks=nb)
    return run, {"bytes": 2 * src.numel() * 2}   # read + write


def case_kv_push_nvlink(dev, tokens=65536, hkv=8, ctas=0, pull=False, ce=False):
    """One layer's KV (64k tokens, 256 MB) from GPU 0's cache into GPU 1's over
    NVLink.  Push: the kernel runs on GPU 0 and stores into GPU 1's memory;
    pull: it runs on GPU 1 and loads GPU 0's memory.  Bytes counted once (the
    bytes that cross the link)."""
    if torch.cuda.device_count() < 2:
        raise SystemExit("kv_push_nvlink needs 2 GPUs")
    bs = 16
    nb = tokens // bs
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    ops.enable_peer_access(0, 1)
    ops.enable_peer_access(1, 0)
    src = torch.randn(2, nb, hkv, bs, 128, device=d0).bfloat16()
    dst = torch.empty_like(src, device=d1)
    run_dev = d1 if pull else d0
    perm = torch.randperm(nb)
    pairs = torch.stack([torch.arange(nb), perm], 1).int().to(run_dev)
    chunk = bs * 128 * 2
    status = ops.new_status(run_dev)
    if ce:
        def run():
            dst.copy_(src, non_blocking=True)
    else:
        def run():
            ops.kv_push_layer(src[0].data_ptr(), src[1].data_ptr(), dst[0].data_ptr(), dst[1].data_ptr(), pairs,
                              src_heads=hkv, dst_heads=hkv, chunk_bytes=chunk, src_blocks=nb, dst_blocks=nb,
                              max_ctas=ctas, status=status)

    def check():
        torch.cuda.synchronize(d0)
        torch.cuda.synchronize(d1)
        if not ce:
            ops.check_status(status, "kv push nvlink")
            got = dst[:, perm.to(d1).long()].float().cpu()
            assert torch.equal(got, src.float().cpu()), "kv_push_nvlink: destination differs from source"
    return run, {"bytes": src.numel() * 2, "device": run_dev, "check": check, "link": True}


def push_beside(dev, co: str = "gemm", ctas: int = 296, tokens: int = 8192, iters: int = 20) -> dict:
    """The KV push of one layer (``tokens`` tokens, local destination) timed
    alone and while another kernel runs on a second stream: ``co`` = gemm
    (the gate/up GEMM of ``tokens`` rows), attn (causal prefill attention of
    4 x ``tokens/4``), or none.  The push runs on a high-priority stream, as
    in the PD prefill; returns per-launch push times (CUDA events)."""
    bs, hkv = 16, 8
    nb = tokens // bs
    src = torch.randn(2, nb, hkv, bs, 128, device=dev).bfloat16()
    dst = torch.empty_like(src)
    pairs = torch.stack([torch.arange(nb), torch.randperm(nb)], 1).int().to(dev)
    status = ops.new_status(dev)
    push_stream = torch.cuda.Stream(device=dev, priority=-1)
    co_stream = torch.cuda.Stream(device=dev)
    if co == "gemm":
        a = torch.randn(tokens, 4096, device=dev).bfloat16()
        w = torch.randn(28672, 4096, device=dev).bfloat16()
        out = torch.empty(tokens, 14336, dtype=torch.bfloat16, device=dev)
        co_fn = lambda: ops.gemm(a, w, out, silu_mul=True)           # noqa: E731
    elif co == "attn":
        qkv = (torch.randn(tokens, 6144, device=dev) * 0.5).bfloat16()
        ti = ops.prefill_tile_info([tokens // 4] * 4, dev)
        ao = torch.empty(tokens, 4096, dtype=torch.bfloat16, device=dev)
        co_fn = lambda: ops.prefill_attention(qkv, ti, 32, 8, ao)     # noqa: E731
    else:
        co_fn = None

    def push():
        ops.kv_push_layer(src[0].data_ptr(), src[1].data_ptr(), dst[0].data_ptr(), dst[1].data_ptr(), pairs,
                          src_heads=hkv, dst_heads=hkv, chunk_bytes=bs * 256, src_blocks=nb, dst_blocks=nb,
                          max_ctas=ctas, status=status)
    times = []
    for i in range(iters + 3):
        torch.cuda.synchronize(dev)
        if co_fn is not None:
            started = torch.cuda.Event()
            with torch.cuda.stream(co_stream):
                co_fn()
                started.record(co_stream)      # the second co-runner launch begins as the push does
                co_fn()
            push_stream.wait_event(started)
        with torch.cuda.stream(push_stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(push_stream)
            push()
            e1.record(push_stream)
        torch.cuda.synchronize(dev)
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    ops.check_status(status, "push beside")
    ms = sorted(times)[len(times) // 2]
    return {"case": "kv_push_beside", "co": co, "ctas": ctas, "tokens": tokens, "ms_p50": round(ms, 4),
            "gbps": round(src.numel() * 2 * 2 / ms / 1e6, 1)}


def case_wsync(dev, layers=2):
    from connex_b200.models.llama import LlamaConfig, random_trainer_weights
    from connex_b200.parallel.wsync import apply_local, engine_manifest, plan_jobs
    cfg = LlamaConfig(layers=layers)
    named = random_trainer_weights(cfg, dev, dtype=torch.float32)
    m = engine_manifest(cfg)
    jobs, _, _ = plan_jobs(cfg, m, named)
    arena = torch.empty(m.total, dtype=torch.uint8, device=dev)
    return (lambda: apply_local(jobs, arena)), {"bytes": m.total * 3}    # 4 B read + 2 B written per element


def case_ep_gemm(dev, T: int = 4096):
    from connex_b200.bench.ep_bench import H, FFN, FusedEP, zipf_routing
    fused = FusedEP(1, 0, dev, T)
    idx, w = zipf_routing(T, seed=3, device=dev)
    x = (torch.randn(T, H, device=dev) * 0.5).bfloat16()
    out = torch.empty_like(x)
    flops = 2 * T * 8 * H * 3 * FFN
    return (lambda: fused.forward(x, idx, w, out)), {"flops": flops}


def case_gemm_m(dev, M=1, N=28672, K=4096, silu=False):
    """A decode-shaped GEMM: M rows against an N x K weight (weight-read bound)."""
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(N, K, device=dev).bfloat16()
    out = torch.empty(M, N // 2 if silu else N, dtype=torch.bfloat16, device=dev)
    return (lambda: ops.gemm(a, b, out, silu_mul=silu)), {"bytes": N * K * 2 + M * K * 2 + M * N * 2}


def case_decode_step(dev, B=1, ctx=1024, graphs=True):
    """One Llama-3-8B decode step for B sequences of ``ctx`` cached tokens,
    replayed from its CUDA graph (device time of the whole step; bytes =
    weights + the KV read)."""
    from connex.pp.handover import CX_CTX, REQUEST_IDS
    from connex_b200.models.llama import LlamaConfig
    from connex_b200.runtime.pp import StageRuntime
    cfg = LlamaConfig.llama3_8b()
    rt = StageRuntime(cfg, 0, cfg.layers, dev, num_blocks=B * (ctx + 64) // 16 + 64, max_tokens=max(B * ctx, 8192),
                      max_batch=B, max_ctx=ctx + 64)
    if graphs:
        rt.enable_decode_graphs()
    rids = [f"r{i}" for i in range(B)]
    ids = torch.randint(16, cfg.vocab_size, (B * ctx,), dtype=torch.int32, device=dev)
    nxt = rt.compute({"kind": "prefill", REQUEST_IDS: rids, CX_CTX: [0] * B, "n_new": [ctx] * B, "ids": ids},
                     [])["next"]
    step = {"kind": "decode", REQUEST_IDS: rids, CX_CTX: [ctx] * B, "n_new": [1] * B, "ids": nxt}
    rt.compute(step, [])
    if graphs:
        fn = rt.graphs[next(b for b in rt.g_buckets if b >= B)][0].replay
    else:
        fn = lambda: rt.compute(step, [])          # noqa: E731 - the same step again, launched eagerly
    weights = sum(t.numel() * 2 for lw in rt.weights.layers for t in (lw.wqkv, lw.wo, lw.w13, lw.w2)) \
        + rt.weights.lm_head.numel() * 2
    kv = B * (ctx + 1) * cfg.kv_bytes_per_token
    return fn, {"bytes": weights + kv}


CASES = {"gemm": lambda d: case_gemm(d), "gemm_qkv": lambda d: case_gemm(d, 8192, 6144, 4096),
         "gemm_silu": lambda d: case_gemm(d, 8192, 28672, 4096, silu=True), "attn": case_attn,
         "attn_paged": case_attn_paged, "attn_t128": lambda d: case_attn(d, tile=128),
         "attn_t256": lambda d: case_attn(d, tile=256),
         "attn_paged_t128": lambda d: case_attn_paged(d, tile=128),
         "attn_paged_t256": lambda d: case_attn_paged(d, tile=256),
         "attn_2x8192_t128": lambda d: case_attn(d, n_seq=2, L=8192, tile=128),
         "attn_2x8192_t256": lambda d: case_attn(d, n_seq=2, L=8192, tile=256),
         "attn_cudnn_2x8192": lambda d: case_attn_library(d, "cudnn", n_seq=2, L=8192), "attn_cudnn": lambda d: case_attn_library(d, "cudnn"),
         "attn_torch_flash": lambda d: case_attn_library(d, "flash"),
         "decode_attn": case_decode_attn, "kv_push": case_kv_push, "wsync": case_wsync, "ep_gemm": case_ep_gemm,
         "ep_t128": lambda d: case_ep_gemm(d, 128),
         "gemm_m1_qkv": lambda d: case_gemm_m(d, 1, 6144, 4096), "gemm_m1_o": lambda d: case_gemm_m(d, 1, 4096, 4096),
         "gemm_m1_gateup": lambda d: case_gemm_m(d, 1, 28672, 4096, silu=True),
         "gemm_m1_down": lambda d: case_gemm_m(d, 1, 4096, 14336),
         "gemm_m32_gateup": lambda d: case_gemm_m(d, 32, 28672, 4096, silu=True),
         "decode_step_b1": lambda d: case_decode_step(d, 1), "decode_step_b32": lambda d: case_decode_step(d, 32),
         "decode_step_b1_eager": lambda d: case_decode_step(d, 1, graphs=False)}
NEEDS_ARGS = {"kv_push_nvlink": case_kv_push_nvlink}


PROF_NAMES = ["mma_wait_q", "mma_wait_k", "mma_wait_v", "mma_wait_p0", "mma_wait_p1", "mma_total",
              "sm0_wait_s", "sm0_softmax", "sm0_epilogue", "sm0_wait_o",
              "sm1_wait_s", "sm1_softmax", "sm1_epilogue", "sm1_wait_o", "producer_wait", "unused"]


def attn_profile(fn, dev) -> dict:
    """One launch of the two-tile prefill attention with its per-CTA cycle
    counters (clock64 of the MMA thread and one lane of each softmax
    warpgroup); returns the mean over CTAs of each counter, in thousands of
    cycles, and each as a share of the MMA thread's total."""
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    buf = torch.zeros(sms * 16, dtype=torch.int64, device=dev)
    ops._C.attention_profile(buf.data_ptr())
    try:
        fn()
        torch.cuda.synchronize(dev)
    finally:
        ops._C.attention_profile(0)
    m = buf.view(sms, 16).double().mean(0).tolist()
    total = m[5] or 1.0
    return {"attn_profile_kcycles": {n: round(v / 1e3, 1) for n, v in zip(PROF_NAMES, m) if n != "unused"},
            "share_of_mma_total": {n: round(v / total, 3) for n, v in zip(PROF_NAMES, m) if n != "unused"}}


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("case", choices=sorted(CASES) + sorted(NEEDS_ARGS) + ["kv_push_beside"])
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--ctas", type=int, default=0, help="kv_push_nvlink: grid size (0 = the launcher's default)")
    p.add_argument("--pull", action="store_true", help="kv_push_nvlink: run on GPU 1, loading GPU 0's memory")
    p.add_argument("--ce", action="store_true", help="kv_push_nvlink: copy-engine peer copy instead of the kernel")
    p.add_argument("--co", default="gemm", help="kv_push_beside: co-running kernel (gemm, attn, none)")
    p.add_argument("--exp-split", type=int, default=None,
                   help="attn cases: softmax exponentials of every 8 on the FMA pipe (0, 2, 4)")
    p.add_argument("--raster-group", type=int, default=None, help="gemm cases: tile-rows per raster band")
    p.add_argument("--attn-profile", action="store_true",
                   help="attn cases: one more launch of the two-tile kernel with its per-CTA cycle counters")
    a = p.parse_args()
    if a.raster_group is not None:
        ops._C.gemm_raster_group(a.raster_group)
    if a.exp_split is not None:
        ops._C.attention_exp_split(a.exp_split)
    dev = torch.device("cuda", 0)
    if a.case == "kv_push_beside":
        print(json.dumps(push_beside(dev, a.co, a.ctas or 296)), flush=True)
        return
    if a.case in NEEDS_ARGS:
        fn, work = NEEDS_ARGS[a.case](dev, ctas=a.ctas, pull=a.pull, ce=a.ce)
    else:
        fn, work = CASES[a.case](dev)
    ms = _time(fn, a.iters, device=work.get("device"))
    if "check" in work:
        work["check"]()
    if a.attn_profile:
        print(json.dumps(attn_profile(fn, dev)), flush=True)
    hbm, tf, src = _peaks()
    res = {"case": a.case, "ms": round(ms, 4)}
    if a.exp_split is not None:
        res["exp_split"] = a.exp_split
    if a.raster_group is not None:
        res["raster_group"] = a.raster_group
    if a.case in NEEDS_ARGS:
        res.update({"ctas": a.ctas, "pull": a.pull, "ce": a.ce})
    if "flops" in work:
        res["tflops"] = round(work["flops"] / ms / 1e9, 1)
        res[f"frac_of_{src}_bf16"] = round(res["tflops"] / tf, 3)
    if "bytes" in work:
        res["gbps"] = round(work["bytes"] / ms / 1e6, 1)
        if work.get("link"):
            # NVLink 5: 770 GB/s measured peer copy per direction on this machine type, 900 nominal
            res["frac_of_770_peer_copy"] = round(res["gbps"] / 770.0, 3)
        else:
            res[f"frac_of_{src}_hbm"] = round(res["gbps"] / hbm, 3)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

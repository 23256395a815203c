"""Device-timed PD-disaggregation benchmark (driven by the repo-root bench.py).

See bench.py for the workload.  Every rank runs the same sequence of
collective steps (barrier, result gathers) in warm-up, timing and error paths.
"""
from __future__ import annotations

import os
import statistics
import time
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

from connex_b200 import ops
from connex_b200.models.llama import LlamaConfig, LlamaModel, LlamaWeights, PagedKVCache
from connex_b200.parallel.peer import PeerHandle, PeerMapper, export_tensor
from connex_b200.runtime.pd import (DecodeBatch, KVDestination, LayerwiseKVPusher, block_pairs,
                                    build_prefill_batch, decode_step)

PUSH_CTAS = 296          # CTAs per layer push (2 per SM): leaves the prefill GEMMs most SMs
TOKEN_BYTES = 64         # first-token inbox copy (16 int32)


def push_ctas(n_pairs: int, n_heads: int) -> int:
    """Launch count of one kv_push_layer (mirrors the host launcher)."""
    warps = n_pairs * 2 * n_heads
    return min((warps + 7) // 8, PUSH_CTAS)


def _prompts(seed: int, step: int, pair: int, batch: int, lo: int, hi: int, vocab: int):
    rng = np.random.default_rng([seed, step, pair])
    lens = rng.integers(lo, hi + 1, size=batch)
    return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens]


def run_pd_bench(args, ClockSampler, finalize: bool = True):
    """The PD steps; with ``finalize=False`` the process group stays up for
    further collective measurements (the caller destroys it)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    if world > 1 and world % 2:
        raise SystemExit("PD bench needs an even number of GPUs (prefill/decode pairs) or 1")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cpu = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
        cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=180))

    def barrier():
        if cpu is not None:
            dist.barrier(group=cpu)

    cfg = LlamaConfig(layers=args.layers)
    role = "both" if world == 1 else ("prefill" if rank < world // 2 else "decode")
    pair = rank if role != "decode" else rank - world // 2
    peer = None if world == 1 else (rank + world // 2 if role == "prefill" else rank - world // 2)
    B = args.batch
    blocks_per_seq = (args.max_len + 1 + cfg.block_size - 1) // cfg.block_size
    n_blocks = 2 * B * blocks_per_seq + 16
    weights = LlamaWeights.random(cfg, dev, seed=args.seed)

    pre = dec = None
    if role in ("prefill", "both"):
        pre_cache = PagedKVCache(cfg, n_blocks, dev)
        pre = LlamaModel(weights, pre_cache, max_tokens=B * args.max_len, max_batch=max(B, 16))
        pusher = LayerwiseKVPusher(pre_cache, max_ctas=PUSH_CTAS)
    if role in ("decode", "both"):
        dec_cache = PagedKVCache(cfg, n_blocks, dev)
        dec = LlamaModel(weights, dec_cache, max_tokens=max(B, 16), max_batch=max(B, 16))
        ready = torch.zeros(16, dtype=torch.int32, device=dev)
        inbox = torch.zeros(TOKEN_BYTES // 4, dtype=torch.int32, device=dev)
        dstatus = ops.new_status(dev)
        ws = ops.decode_workspace(B, cfg.heads, args.max_len + 2, dev)
        tok_host = torch.zeros(B, dtype=torch.int32).pin_memory()

    # ---- peer mapping of the decode caches (control plane: object gather) ----
    mapper = PeerMapper(local)
    if world == 1:
        dst = KVDestination.of_cache(dec_cache, ready)
        inbox_addr = inbox.data_ptr()
    else:
        mine = None
        if role == "decode":
            mine = {"kv": export_tensor(dec_cache.kv).to_dict(), "ready": export_tensor(ready).to_dict(),
                    "inbox": export_tensor(inbox).to_dict(), "blocks": n_blocks,
                    "layer_stride": dec_cache.layer_stride_bytes, "kv_stride": dec_cache.kv_stride_bytes}
        allx = [None] * world
        dist.all_gather_object(allx, mine, group=cpu)
        if role == "prefill":
            d = allx[peer]
            base = mapper.open(PeerHandle.from_dict(d["kv"]))
            dst = KVDestination(base=base, layer_stride=d["layer_stride"], kv_stride=d["kv_stride"],
                                heads=cfg.kv_heads, num_blocks=d["blocks"],
                                ready_addr=mapper.open(PeerHandle.from_dict(d["ready"])))
            inbox_addr = mapper.open(PeerHandle.from_dict(d["inbox"]))
    ready_target = 0
    tok_seg = None

    def run_step(step: int, timed: bool):
        nonlocal ready_target, tok_seg
        prompts = _prompts(args.seed, step, pair, B, args.min_len, args.max_len, cfg.vocab_size)
        lens = [len(p) for p in prompts]
        n_pairs_total = sum((n + cfg.block_size - 1) // cfg.block_size for n in lens)
        # destination blocks: allocated by the decode instance, sent to its prefill peer
        dblocks = None
        if role in ("decode", "both"):
            dblocks = [dec_cache.allocate(dec_cache.blocks_needed(n + 1)) for n in lens]
        if role == "decode":
            dist.send_object_list([dblocks], dst=peer, group=cpu)
        elif role == "prefill":
            box = [None]
            dist.recv_object_list(box, src=peer, group=cpu)
            dblocks = box[0]
        ids_host = torch.tensor([t for p in prompts for t in p], dtype=torch.int32).pin_memory()
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = ops.launch_count()
        e0.record()
        push_ms = 0.0
        kv_bytes = 0
        if role in ("prefill", "both"):
            ids = ids_host.to(dev, non_blocking=True)                      # H2D from pinned memory
            batch = build_prefill_batch(pre.cache, prompts, dev, ids=ids)
            pairs = block_pairs(batch.src_blocks, [d[:len(s)] for d, s in zip(dblocks, batch.src_blocks)], dev)
            pusher.begin(pairs, dst, timing=True)
            nxt = pre.prefill(batch.ids, batch.positions, batch.slots, batch.seq_lens, batch.last_rows,
                              batch.tile_info, layer_hook=pusher.hook)
            # first tokens -> decode inbox, on the push stream after the prefill's head
            pusher.stream.wait_stream(torch.cuda.current_stream(dev))
            if tok_seg is None:
                tok_seg = torch.tensor([[pre.next_ids.data_ptr(), inbox_addr, TOKEN_BYTES]],
                                       dtype=torch.int64, device=dev)
            with torch.cuda.stream(pusher.stream):
                ops.copy_segments(tok_seg, TOKEN_BYTES, ready=dst.ready_addr, max_ctas=1, status=pusher.status)
            pusher.join()
            kv_bytes = pusher.bytes  # summed over all layers
        if role in ("decode", "both"):
            ready_target += cfg.layers * push_ctas(n_pairs_total, cfg.kv_heads) + 1
            ops.wait_flag(ready.data_ptr(), ready_target, dstatus, timeout_s=30.0)
            db = DecodeBatch(dec_cache, dblocks, lens, dev)
            tok = decode_step(dec, db, inbox[:B], ws)
            tok_host.copy_(tok[:B], non_blocking=True)                     # D2H of the step's result
        e1.record()
        torch.cuda.synchronize(dev)
        launches = ops.launch_count() - l0
        step_ms = e0.elapsed_time(e1)
        if role in ("prefill", "both"):
            push_ms = pusher.push_ms()
            ops.check_status(pusher.status, "kv push")
            for b in batch.src_blocks:
                pre.cache.free(b)
        if role in ("decode", "both"):
            ops.check_status(dstatus, "decode wait")
            for b in dblocks:
                dec_cache.free(b)
        return {"step_ms": step_ms, "push_ms": push_ms, "kv_bytes": kv_bytes, "tokens": sum(lens),
                "launches": launches, "lens": lens}

    for w in range(args.warmup):
        run_step(10_000 + w, False)
    clocks = ClockSampler(range(torch.cuda.device_count())) if local == 0 else None
    if clocks:
        clocks.start()
    recs = [run_step(s, True) for s in range(args.steps)]
    clk = clocks.stop() if clocks else None

    gathered = [None] * world
    if world > 1:
        dist.all_gather_object(gathered, {"role": role, "recs": recs, "clk": clk}, group=cpu)
    else:
        gathered = [{"role": role, "recs": recs, "clk": clk}]
    result = None
    if rank == 0:
        K = args.steps
        step_max = [max(g["recs"][s]["step_ms"] for g in gathered) for s in range(K)]
        prod = [g for g in gathered if g["role"] in ("prefill", "both")]
        kv_total = sum(g["recs"][s]["kv_bytes"] for g in prod for s in range(K))
        push_max = [max(g["recs"][s]["push_ms"] for g in prod) for s in range(K)]
        push_sum_by_pair = [sum(g["recs"][s]["push_ms"] for s in range(K)) for g in prod]
        kv_by_pair = [sum(g["recs"][s]["kv_bytes"] for s in range(K)) for g in prod]
        # aggregate bandwidth of the push kernels: sum over pairs of bytes / device time
        value = sum(b / (t * 1e-3) for b, t in zip(kv_by_pair, push_sum_by_pair)) / 1e9
        e2e = kv_total / (sum(step_max) * 1e-3) / 1e9
        tokens = sum(g["recs"][s]["tokens"] for g in prod for s in range(K))
        launches = sum(g["recs"][s]["launches"] for g in gathered for s in range(K))
        clk0 = gathered[0]["clk"] or {}
        result = {
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(step_max), 3),
            "p50_ttft_ms": round(statistics.median(step_max), 3),
            "kv_bytes_per_step": kv_total // K,
            "push_ms_per_step_max": round(statistics.mean(push_max), 3),
            "prefill_tokens_per_s": round(tokens / (sum(step_max) * 1e-3), 1),
            "e2e": {"value": round(e2e, 3), "unit": "GB/s KV delivered (whole step, public PD API)",
                    "h2d_bytes_per_step": 4 * tokens // K, "d2h_bytes_per_step": 4 * B * len(prod)},
            "gpu_launches": launches,
            "clocks": {"sm_mhz": clk0.get("sm_mhz"), "sm_max_mhz": clk0.get("sm_max_mhz"),
                       "reasons": clk0.get("reasons", [])},
            "data": "synthetic (random token ids, random-init N(0,0.02) weights, seed 0)",
            "config": {"model": f"Llama-3-8B architecture ({cfg.layers} layers)", "global_batch": B * len(prod),
                       "seq_len": f"uniform {args.min_len}-{args.max_len}",
                       "parallelism": "colocated 1P1D" if world == 1 else f"pd {world // 2}P{world // 2}D (TP1)",
                       "kv_block_tokens": cfg.block_size, "l2": "inputs larger than L2 (16 GB weights, GB-scale KV)"},
        }
    if world > 1:
        barrier()
        mapper.close()
        if finalize:
            dist.destroy_process_group()
    return result

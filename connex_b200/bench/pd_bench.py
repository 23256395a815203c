"""Device-timed PD-disaggregation benchmark (driven by the repo-root bench.py).

See bench.py for the workload.  Every rank runs the same sequence of
collective steps (barrier, result gathers) in warm-up, timing and error paths.
"""
from __future__ import annotations

import os
import statistics
from datetime import timedelta
from typing import Sequence

import numpy as np
import torch
import torch.distributed as dist

from connex_b200 import ops
from connex_b200.models.llama import LlamaConfig, LlamaModel, LlamaWeights, PagedKVCache
from connex_b200.parallel.peer import PeerHandle, PeerMapper, export_tensor
from connex_b200.runtime.pd import (DecodeBatch, KVDestination, LayerReadySignal, LayerwiseKVPuller,
                                    LayerwiseKVPusher, block_pairs, build_prefill_batch, decode_step)

PUSH_CTAS = int(os.environ.get("CX_PD_PUSH_CTAS", "0"))   # CTAs per layer push (0: one 128-thread CTA per SM)
PUSH_AFTER_ATTENTION = os.environ.get("CX_PD_PUSH_AFTER", "kv") == "attention"
PULL_CTAS = int(os.environ.get("CX_PD_PULL_CTAS", "592"))   # the decode GPU is otherwise idle during prefill
TOKEN_BYTES = 64         # first-token inbox copy (16 int32)


def push_ctas(n_pairs: int, n_heads: int) -> int:
    """Launch count of one kv_push_layer (mirrors the host launcher)."""
    warps = n_pairs * 2 * n_heads
    return min((warps + 7) // 8, PUSH_CTAS)


def _prompts(seed: int, step: int, batch: int, lo: int, hi: int, vocab: int):
    """The step's prompts.  Every prefill/decode pair draws the same lengths in
    a step, so the max-over-ranks step time measures the transfer, not the
    slowest random draw."""
    rng = np.random.default_rng([seed, step])
    lens = rng.integers(lo, hi + 1, size=batch)
    return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens]


def _runs(src: Sequence[int], dst: Sequence[int]):
    """(src0, dst0, n) runs where both block lists advance by one."""
    out = []
    for s, d in zip(src, dst):
        if out and out[-1][0] + out[-1][2] == s and out[-1][1] + out[-1][2] == d:
            out[-1][2] += 1
        else:
            out.append([s, d, 1])
    return [tuple(r) for r in out]


def kv_checksum(cache: PagedKVCache, blocks: Sequence[Sequence[int]], lens: Sequence[int]) -> list:
    """Order-sensitive checksums of each request's first ``n`` cached tokens
    over all layers: the sum and the token-position-weighted sum in fp64."""
    out = []
    for b, n in zip(blocks, lens):
        nb = (n + cache.cfg.block_size - 1) // cache.cfg.block_size
        idx = torch.tensor(list(b[:nb]), dtype=torch.long, device=cache.kv.device)
        x = cache.kv.index_select(2, idx)                             # [L, 2, nb, H, BS, D]
        L, two, _, H, BS, D = x.shape
        x = x.permute(0, 1, 3, 2, 4, 5).reshape(L, two, H, nb * BS, D)[:, :, :, :n].double()
        w = torch.arange(1, n + 1, dtype=torch.float64, device=x.device).view(1, 1, 1, -1, 1)
        out.append((round(float(x.sum()), 6), round(float((x * w).sum()), 6)))
    return out


def _job_gpu_uuids(world: int, cpu, dev) -> list:
    """UUIDs of the GPUs this job's ranks drive (nvidia-smi ``uuid`` form)."""
    mine = str(torch.cuda.get_device_properties(dev).uuid)
    mine = mine if mine.startswith("GPU-") else "GPU-" + mine
    if world == 1:
        return [mine]
    allu = [None] * world
    dist.all_gather_object(allu, mine, group=cpu)
    return allu


def kv_mode(args, world: int) -> str:
    """The layerwise transfer the timed steps use: ``--kv-mode`` (or
    ``CX_PD_KV_MODE``); by default pull between GPUs, push on one GPU."""
    m = getattr(args, "kv_mode", None) or os.environ.get("CX_PD_KV_MODE") or "auto"
    if m == "auto":
        m = "pull" if world > 1 else "push"
    if m not in ("push", "pull"):
        raise SystemExit(f"kv mode must be push, pull or auto, got {m!r}")
    return "push" if world == 1 else m


def _pair_rate(ranks: list, key: str, n: int, field: str) -> float:
    """Aggregate GB/s: sum over the transferring ranks of bytes / summed time."""
    total = 0.0
    for g in ranks:
        b = sum(g[key][s]["kv_bytes"] for s in range(n))
        t = sum(g[key][s][field] for s in range(n))
        if t > 0:
            total += b / (t * 1e-3)
    return total / 1e9


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
        layer_ctr = torch.zeros(4, dtype=torch.int32, device=dev)      # pull mode: prefill's per-layer counter
        puller = LayerwiseKVPuller(dec_cache, max_ctas=PULL_CTAS)

    # ---- peer mapping of the decode caches (control plane: object gather) ----
    mapper = PeerMapper(local)
    signal = None
    if world == 1:
        dst = KVDestination.of_cache(dec_cache, ready)
        inbox_addr = inbox.data_ptr()
    else:
        mine = None
        if role == "decode":
            mine = {"kv": export_tensor(dec_cache.kv).to_dict(), "ready": export_tensor(ready).to_dict(),
                    "inbox": export_tensor(inbox).to_dict(), "layer_ctr": export_tensor(layer_ctr).to_dict(),
                    "blocks": n_blocks, "layer_stride": dec_cache.layer_stride_bytes,
                    "kv_stride": dec_cache.kv_stride_bytes}
        else:
            mine = {"kv": export_tensor(pre_cache.kv).to_dict(), "blocks": n_blocks,
                    "layer_stride": pre_cache.layer_stride_bytes, "kv_stride": pre_cache.kv_stride_bytes}
        allx = [None] * world
        dist.all_gather_object(allx, mine, group=cpu)
        d = allx[peer]
        if role == "prefill":
            base = mapper.open(PeerHandle.from_dict(d["kv"]))
            dst = KVDestination(base=base, layer_stride=d["layer_stride"], kv_stride=d["kv_stride"],
                                heads=cfg.kv_heads, num_blocks=d["blocks"],
                                ready_addr=mapper.open(PeerHandle.from_dict(d["ready"])))
            inbox_addr = mapper.open(PeerHandle.from_dict(d["inbox"]))
            signal = LayerReadySignal(mapper.open(PeerHandle.from_dict(d["layer_ctr"])), dev, cfg.layers)
        else:
            src_view = {"base": mapper.open(PeerHandle.from_dict(d["kv"])), "blocks": d["blocks"],
                        "layer_stride": d["layer_stride"], "kv_stride": d["kv_stride"]}
    ready_target = 0
    pull_base = 0
    tok_seg = None

    def run_step(step: int, timed: bool, check: bool = False, mode: str = "push"):
        """One step.  ``mode``: ``push`` (the prefill GPU's kernel stores each
        layer into the decode cache), ``pull`` (the decode GPU's kernel
        gathers each layer as soon as the prefill publishes it), or ``bulk``
        (the reference's design: prefill every layer, then copy the whole KV
        with one copy-engine peer copy per (layer, K/V, run of consecutive
        blocks)).  ``check``: after the step, compare checksums of the
        prefill side's source blocks and the decode side's destination blocks
        (outside any timed region)."""
        nonlocal ready_target, tok_seg, pull_base
        bulk = mode == "bulk"
        pull = mode == "pull" and world > 1
        prompts = _prompts(args.seed, step, B, args.min_len, args.max_len, cfg.vocab_size)
        lens = [len(p) for p in prompts]
        n_pairs_total = sum((n + cfg.block_size - 1) // cfg.block_size for n in lens)
        # destination blocks: allocated by the decode instance, sent to its prefill peer
        dblocks = None
        if role in ("decode", "both"):
            dblocks = [dec_cache.allocate(dec_cache.blocks_needed(n + 1)) for n in lens]
        sblocks = None
        if pull and role == "prefill":       # source blocks are allocated up front so the puller knows them
            sblocks = [pre.cache.allocate(pre.cache.blocks_needed(n)) for n in lens]
        if role == "decode":
            dist.send_object_list([dblocks], dst=peer, group=cpu)
            if pull:
                box = [None]
                dist.recv_object_list(box, src=peer, group=cpu)
                sblocks = box[0]
        elif role == "prefill":
            box = [None]
            dist.recv_object_list(box, src=peer, group=cpu)
            dblocks = box[0]
            if pull:
                dist.send_object_list([sblocks], dst=peer, group=cpu)
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
            batch = build_prefill_batch(pre.cache, prompts, dev, ids=ids, blocks=sblocks)
            pairs = block_pairs(batch.src_blocks, [d[:len(s)] for d, s in zip(dblocks, batch.src_blocks)], dev)
            hook = None
            if pull:
                hook = signal.hook
            elif not bulk:
                pusher.begin(pairs, dst, timing=True)
                hook = pusher.hook
            nxt = pre.prefill(batch.ids, batch.positions, batch.slots, batch.seq_lens, batch.last_rows,
                              batch.tile_info, layer_hook=hook, hook_after_attention=PUSH_AFTER_ATTENTION)
            if pull:
                signal.end()
            # first tokens -> decode inbox, on the push stream after the prefill's head
            pusher.stream.wait_stream(torch.cuda.current_stream(dev))
            if tok_seg is None:
                tok_seg = torch.tensor([[pre.next_ids.data_ptr(), inbox_addr, TOKEN_BYTES]],
                                       dtype=torch.int64, device=dev)
            with torch.cuda.stream(pusher.stream):
                if bulk:
                    kv_bytes = bulk_copy(batch.src_blocks, dblocks)
                ops.copy_segments(tok_seg, TOKEN_BYTES, ready=dst.ready_addr, max_ctas=1, status=pusher.status)
            pusher.join()
            if mode == "push":
                kv_bytes = pusher.bytes  # summed over all layers
        if role in ("decode", "both"):
            if pull:
                pairs_d = block_pairs(sblocks, [d[:len(s)] for d, s in zip(dblocks, sblocks)], dev)
                puller.pull(src_view["base"], src_view["layer_stride"], src_view["kv_stride"], cfg.kv_heads,
                            src_view["blocks"], pairs_d, layer_ctr.data_ptr(), pull_base, timing=True)
                pull_base += cfg.layers
                kv_bytes = puller.bytes
            ready_target += (cfg.layers * push_ctas(n_pairs_total, cfg.kv_heads) if mode == "push" else 0) + 1
            ops.wait_flag(ready.data_ptr(), ready_target, dstatus, timeout_s=30.0)
            db = DecodeBatch(dec_cache, dblocks, lens, dev)
            tok = decode_step(dec, db, inbox[:B], ws)
            tok_host.copy_(tok[:B], non_blocking=True)                     # D2H of the step's result
        e1.record()
        torch.cuda.synchronize(dev)
        launches = ops.launch_count() - l0
        step_ms = e0.elapsed_time(e1)
        sums = None
        if check:
            sums = {}
            if role in ("prefill", "both"):
                sums["src"] = kv_checksum(pre.cache, batch.src_blocks, lens)
            if role in ("decode", "both"):
                sums["dst"] = kv_checksum(dec_cache, dblocks, lens)
        kernel_ms = 0.0
        if role in ("prefill", "both"):
            if mode == "push":
                push_ms, kernel_ms = pusher.push_ms(), pusher.kernel_ms()
            ops.check_status(pusher.status, "kv push")
            for b in batch.src_blocks:
                pre.cache.free(b)
        if role in ("decode", "both"):
            if pull:
                push_ms, kernel_ms = puller.pull_ms(), puller.kernel_ms()
                ops.check_status(puller.status, "kv pull")
            ops.check_status(dstatus, "decode wait")
            for b in dblocks:
                dec_cache.free(b)
        # the rank that ran the transfer kernels reports their bytes and times
        mover = (role == "decode") if pull else (role in ("prefill", "both"))
        return {"step_ms": step_ms, "push_ms": push_ms if mover else 0.0, "kernel_ms": kernel_ms if mover else 0.0,
                "kv_bytes": kv_bytes if mover else 0, "tokens": sum(lens) if role != "decode" else 0,
                "launches": launches, "lens": lens, "sums": sums, "mover": mover}

    def bulk_copy(src_blocks, dst_blocks) -> int:
        """The reference's design: after the whole prefill, copy every layer's
        K and V block runs with the copy engine (one memcpy per run)."""
        nbytes = 0
        hs = pre.cache.head_slice_bytes * cfg.kv_heads          # one block of one layer's K (or V)
        for sb, db in zip(src_blocks, dst_blocks):
            for s0, d0, n in _runs(sb, db[:len(sb)]):
                for layer in range(cfg.layers):
                    for kv in range(2):
                        src = pre.cache.kv[layer, kv, s0:s0 + n]
                        dptr = dst.base + layer * dst.layer_stride + kv * dst.kv_stride + d0 * hs
                        ops.from_ptr(dptr, list(src.shape), src.dtype, dev.index).copy_(src, non_blocking=True)
                        nbytes += n * hs
        return nbytes

    mode = kv_mode(args, world)
    other = "push" if mode == "pull" else None
    for w in range(args.warmup):
        run_step(10_000 + w, False, mode=mode)
    sampled = _job_gpu_uuids(world, cpu, dev)
    clocks = ClockSampler(sampled) if local == 0 else None
    if clocks:
        clocks.start()
    recs = [run_step(s, True, mode=mode) for s in range(args.steps)]
    clk = clocks.stop() if clocks else None
    # outside the timed region: KV checksum of one step, the other layerwise
    # mode on the same prompts, and the bulk-copy design (TTFT comparison)
    chk = run_step(20_000, False, check=True, mode=mode)
    n_cmp = max(3, min(args.steps, 8))
    alt = []
    if other is not None:
        run_step(40_000, False, mode=other)
        alt = [run_step(s, False, mode=other) for s in range(n_cmp)]
    run_step(30_000, False, mode="bulk")
    bulk = [run_step(s, False, mode="bulk") for s in range(n_cmp)]

    gathered = [None] * world
    mine = {"role": role, "recs": recs, "clk": clk, "sums": chk["sums"], "bulk": bulk, "alt": alt}
    if world > 1:
        dist.all_gather_object(gathered, mine, group=cpu)
    else:
        gathered = [mine]
    result = None
    if rank == 0:
        K = args.steps
        step_max = [max(g["recs"][s]["step_ms"] for g in gathered) for s in range(K)]
        prod = [g for g in gathered if g["role"] in ("prefill", "both")]
        movers = [g for g in gathered if g["recs"][0]["mover"]]      # the ranks that ran the KV kernels
        kv_total = sum(g["recs"][s]["kv_bytes"] for g in movers for s in range(K))
        push_max = [max(g["recs"][s]["push_ms"] for g in movers) for s in range(K)]
        value = _pair_rate(movers, "recs", K, "push_ms")
        window_gbps = _pair_rate(movers, "recs", K, "kernel_ms")
        e2e = kv_total / (sum(step_max) * 1e-3) / 1e9
        tokens = sum(g["recs"][s]["tokens"] for g in gathered for s in range(K))
        launches = sum(g["recs"][s]["launches"] for g in gathered for s in range(K))
        clk0 = gathered[0]["clk"] or {}
        # KV check: every pair's decode-side blocks equal its prefill-side blocks
        if world == 1:
            ok = gathered[0]["sums"]["src"] == gathered[0]["sums"]["dst"]
        else:
            ok = all(gathered[r]["sums"]["src"] == gathered[r + world // 2]["sums"]["dst"] for r in range(world // 2))
        bulk_max = [max(g["bulk"][s]["step_ms"] for g in gathered) for s in range(n_cmp)]
        alt_stats = {}
        if alt:
            alt_movers = [g for g in gathered if g["alt"][0]["mover"]]
            alt_max = [max(g["alt"][s]["step_ms"] for g in gathered) for s in range(n_cmp)]
            alt_stats = {f"kv_{other}_gbps": round(_pair_rate(alt_movers, "alt", n_cmp, "push_ms"), 2),
                         f"kv_{other}_kernel_window_gbps": round(_pair_rate(alt_movers, "alt", n_cmp, "kernel_ms"), 2),
                         f"p50_ttft_ms_{other}": round(statistics.median(alt_max), 3)}
        result = {
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(step_max), 3),
            "p50_ttft_ms": round(statistics.median(step_max), 3),
            "kv_bytes_per_step": kv_total // K,
            "kv_ms_per_step_max": round(statistics.mean(push_max), 3),
            # the same bytes over the transfer kernels' own execution windows
            # (%globaltimer, first CTA start to last CTA end): launch and
            # queueing delays on the transfer stream excluded
            "kv_kernel_window_gbps": round(window_gbps, 2),
            "prefill_tokens_per_s": round(tokens / (sum(step_max) * 1e-3), 1),
            "kv_check": "ok" if ok else "MISMATCH",
            "kv_transfer": ("pull: the decode GPU's kernel gathers each layer from the prefill GPU's cache over "
                            "NVLink as soon as the prefill publishes it" if mode == "pull" else
                            "push: the prefill GPU's kernel stores each layer into the decode cache right after "
                            "the layer's KV write"),
            **alt_stats,
            "p50_ttft_ms_bulk_copy_after_prefill": round(statistics.median(bulk_max), 3),
            "e2e": {"value": round(e2e, 3),
                    "unit": ("GB/s of KV delivered per second of the whole step through connex_b200.runtime.pd "
                             f"(H2D of prompt ids, prefill with the layerwise {mode}, decode first token, D2H)"),
                    "h2d_bytes_per_step": 4 * tokens // K, "d2h_bytes_per_step": 4 * B * len(prod)},
            "gpu_launches": launches,
            "clocks": {"sm_mhz": clk0.get("sm_mhz"), "sm_max_mhz": clk0.get("sm_max_mhz"),
                       "reasons": clk0.get("reasons", [])},
            "data": "synthetic (random token ids, random-init N(0,0.02) weights, seed 0)",
            "config": {"model": f"Llama-3-8B architecture ({cfg.layers} layers)", "global_batch": B * len(prod),
                       "seq_len": f"uniform {args.min_len}-{args.max_len}",
                       "parallelism": "colocated 1P1D" if world == 1 else f"pd {world // 2}P{world // 2}D (TP1)",
                       "kv_block_tokens": cfg.block_size, "l2": "inputs larger than L2 (16 GB weights, GB-scale KV)",
                       "kv_ctas": PULL_CTAS if mode == "pull" else (PUSH_CTAS or "one 128-thread CTA per SM"),
                       "push_after": "attention" if PUSH_AFTER_ATTENTION else "kv write"},
        }
    if rank == 0 and result is not None and result["kv_check"] != "ok":
        raise SystemExit("kv_check failed: decode-side KV differs from the prefill side")
    if world > 1:
        barrier()
        mapper.close()
        if finalize:
            dist.destroy_process_group()
    return result

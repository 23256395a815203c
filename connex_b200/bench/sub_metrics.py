"""Secondary metrics of the flagship benchmark line, measured in the same job
right after the PD steps: the fused Llama-3-8B weight broadcast (fp32
trainer weights -> bf16 engine layout on every other GPU) against an NCCL
broadcast (and, N >= 4, from two FSDP trainer shards on ranks 0-1 to the
other GPUs, against NCCL broadcasts of the cast shards), the fused EP MoE
layer latency (dispatch + expert GEMMs +
combine, Qwen3-30B-A3B layer geometry, 128 tokens per rank) with its
per-phase split, against the NCCL all-to-all baseline with grouped expert
GEMMs, and (N > 1) the EP failover time: the last rank
leaves, the others route around it and finish their next forward (host
clock of the box).  The rest are device-timed, max over ranks.  Every rank
must call :func:`run_sub_metrics` (it is collective when N > 1).
"""
from __future__ import annotations

from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as dist


def run_sub_metrics(world: int, rank: int, dev, layers: int = 32) -> Optional[dict]:
    from connex_b200.bench.ep_bench import reduce_max, run_ep_bench
    from connex_b200.bench.wsync_bench import run as run_wsync
    from connex_b200.models.llama import LlamaConfig
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=180)) if world > 1 else None
    ws = run_wsync(LlamaConfig(layers=layers), iters=3, warmup=2)
    torch.cuda.empty_cache()
    wsh = None
    if world >= 4:        # the RL config's shape: FSDP trainer shards on ranks 0-1, rollouts on the rest
        from connex_b200.bench.wsync_bench import run_sharded
        wsh = run_sharded(LlamaConfig(layers=layers), trainers=2, iters=3, warmup=2)
        torch.cuda.empty_cache()
    ep = run_ep_bench(world, rank, dev, cpu, None, tokens=(128,), iters=10, warmup=3, failover=True)
    torch.cuda.empty_cache()
    allr = [ep]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, ep, group=cpu)
    if rank != 0:
        return None
    e = reduce_max(allr)["128"]
    out = {"ep_layer_us_t128": e["cx_us"], "ep_layer_us_t128_nccl_baseline": e["nccl_us"],
           "ep_layer_phases_us_t128": {p: e.get(f"phase_{p}_us") for p in ("count", "dispatch", "gate_up", "down",
                                                                           "combine")},
           "weight_sync_bytes": ws["engine_bytes"]}
    if world > 1:
        out["ep_failover_ms"] = round(max(r.get("failover_ms", 0.0) for r in allr), 2)
    if world == 1:
        out["weight_convert_ms_local"] = round(ws["local_ms"], 3)
    else:
        for k in ("fused_multicast_ms", "fused_relay_ms", "fused_relay_p2p_ms", "fused_p2p_ms", "nccl_ms"):
            if ws.get(k) is not None:
                out[f"weight_sync_{k}"] = round(ws[k], 3)
        if wsh is not None:
            for k in ("fused_multicast_ms", "nccl_ms"):
                if wsh.get(k) is not None:
                    out[f"weight_sync_fsdp2_{k}"] = round(wsh[k], 3)
    return out

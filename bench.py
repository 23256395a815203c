#!/usr/bin/env python
"""Flagship benchmark: PD-disaggregated serving of Llama-3-8B (bf16, random init).

One step = each prefill instance takes a batch of prompts (lengths drawn
uniformly from 512..8192, random token ids over the 128256-entry vocab),
prefills them with the native tcgen05 runtime while the fused
``kv_push_layer`` kernel pushes each layer's paged KV (16-token blocks,
32 layers x 8 KV heads x 128, bf16) into the decode instance's cache over
NVLink peer memory, then the decode instance acquire-waits on the device
ready counter and produces the first output token.

Topology: N = 1 runs a prefill and a decode instance on the same GPU (the
push is a local copy); N >= 2 runs N/2 prefill GPUs -> N/2 decode GPUs,
pairwise (config: 4 prefill -> 4 decode at N = 8).  Per-pair work is fixed
(weak scaling).

Reported (rank 0, one JSON line):
* ``value``     -- aggregate KV transfer bandwidth of the push kernels
                   (bytes / summed device time of the push launches, summed
                   over pairs), GB/s;
* ``e2e``       -- KV bytes delivered per second of the whole step, measured
                   through the public PD API including the H2D copy of the
                   prompt ids from pinned memory and the D2H read of the
                   first tokens;
* ``p50_ttft_ms``, per-step times, clocks and launch counts;
* ``sub_metrics`` -- the fused EP MoE layer and the fused weight broadcast
  (each against its NCCL baseline), the EP failover time, and (N >= 2) a
  10-second serving run per pair under Poisson load (4 requests/s, 128
  output tokens): ``serving_ttft_p50_ms``, ``serving_tpot_p50_ms``, ...

Timing: W untimed warm-up steps, then K steps, each bracketed by a barrier
and ``torch.cuda.synchronize()``; device time by CUDA events; max over ranks.
Inputs (16 GB of weights, GBs of KV per step) exceed the 126 MB L2.

``--impl reference`` runs the unmodified reference (HeterInfra/connex) when
it can move GPU KV on this machine; otherwise it prints an ``unavailable`` line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PUBLISHED_KV_GBPS = 9.8  # reference: 128 MB prompt KV in ~13 ms (docs/results.md:869-871)
METRIC = "PD KV GB/s + p50 TTFT; EP dispatch+combine µs; weight-sync s; failover ms"


def reference_arm(args) -> None:
    """The reference's own PD KV hand-off on this machine (see
    ``connex_b200/bench/reference_pd.py``): its ``KVProducer.hold`` /
    ``KVConsumer.pull`` with the data plane its stock selection takes here
    (pinned host staging over the in-process loopback plane; connex-rs and
    Mooncake are not installed).  One pair per prefill rank: rank r's
    process drives GPU r (prefill cache) and GPU r + N/2 (decode cache);
    N = 1 keeps both caches on GPU 0.  Host clock around each hand-off
    (the reference's data plane here is host code), max over pairs."""
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ref = os.path.join(ROOT, "baseline", "_ref")

    def say(obj):
        if rank == 0:
            print(json.dumps(obj), flush=True)
    if not os.path.isdir(os.path.join(ref, "connex")):
        say({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"})
        return
    if world > 1 and world % 2:
        say({"impl": "reference", "unavailable": "needs an even number of GPUs (prefill/decode pairs)"})
        return
    import torch
    cpu = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=900))
        cpu = dist.group.WORLD
    mover = world == 1 or rank < world // 2
    src, dst = (local, local if world == 1 else local + world // 2)
    uuids = []
    for d in sorted({src, dst}):
        u = str(torch.cuda.get_device_properties(d).uuid)
        uuids.append(u if u.startswith("GPU-") else "GPU-" + u)
    out, err, clk = None, None, None
    if mover:
        cmd = [sys.executable, "-I", os.path.join(ROOT, "connex_b200", "bench", "reference_pd.py"), "--ref", ref,
               "--src-device", str(src), "--dst-device", str(dst), "--steps", str(args.steps),
               "--warmup", str(args.warmup), "--batch", str(args.batch), "--min-len", str(args.min_len),
               "--max-len", str(args.max_len), "--layers", str(args.layers), "--seed", str(args.seed)]
        clocks = ClockSampler(uuids)
        clocks.start()
        r = subprocess.run(cmd, capture_output=True, text=True, cwd="/tmp", timeout=1800)
        clk = clocks.stop()
        lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
        if r.returncode != 0 or not lines:
            err = (r.stderr.strip().splitlines() or ["no output"])[-1][:300]
        else:
            out = json.loads(lines[-1])
    allr = [{"out": out, "err": err, "clk": clk, "mover": mover}]
    if world > 1:
        import torch.distributed as dist
        allr = [None] * world
        dist.all_gather_object(allr, {"out": out, "err": err, "clk": clk, "mover": mover}, group=cpu)
        dist.destroy_process_group()
    if rank != 0:
        return
    errs = [x["err"] for x in allr if x["mover"] and x["err"]]
    if errs:
        say({"impl": "reference", "unavailable": f"reference PD hand-off failed on this machine: {errs[0]}"})
        return
    runs = [x["out"] for x in allr if x["mover"]]
    K = args.steps
    value = sum(sum(r["bytes"] for r in o["recs"]) / sum(r["pull_s"] for r in o["recs"]) for o in runs) / 1e9
    step_max = [max(o["recs"][s]["step_s"] for o in runs) for s in range(K)]
    kv_total = sum(r["bytes"] for o in runs for r in o["recs"])
    clk0 = allr[0]["clk"] or {}
    say({"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
         "steps": K, "warmup": args.warmup, "ms_per_step": round(1e3 * statistics.mean(step_max), 3),
         "higher_is_better": True, "scaling": "weak",
         "vs_baseline": round(value / PUBLISHED_KV_GBPS, 3),
         "e2e": {"value": round(kv_total / sum(step_max) / 1e9, 3),
                 "unit": "GB/s of KV delivered per second of hand-off (hold incl. device->host staging, "
                         "until every pull is back on the decode GPU)",
                 "h2d_bytes_per_step": kv_total // K, "d2h_bytes_per_step": kv_total // K},
         "kv_check": "ok" if all(o["kv_check"] for o in runs) else "MISMATCH",
         "kv_bytes_per_step": kv_total // K,
         "gpu_launches": 0,
         "clocks": {"sm_mhz": clk0.get("sm_mhz"), "sm_max_mhz": clk0.get("sm_max_mhz"),
                    "reasons": clk0.get("reasons", [])},
         "dtype": "bf16", "data": "synthetic (random KV contents; prompt lengths drawn as in the flagship, seed 0)",
         "timing": "host clock (the reference's data plane on this machine is host code); max over pairs",
         "config": {"model": f"Llama-3-8B KV geometry ({args.layers} layers x 8 KV heads x 128, 16-token blocks)",
                    "global_batch": args.batch * len(runs), "seq_len": f"uniform {args.min_len}-{args.max_len}",
                    "parallelism": "colocated 1P1D" if world == 1 else f"pd {world // 2}P{world // 2}D (TP1)",
                    "data_plane": "reference KVProducer/KVConsumer, host staging + in-process loopback plane "
                                  "(connex-rs / Mooncake not installed, no GPUDirect peer-memory driver)",
                    "l2": "inputs larger than L2 (GB-scale KV)"}})


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region, on
    this job's GPUs only (``gpus``: their UUIDs, ``GPU-...`` as nvidia-smi
    prints them)."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = {str(g).lower() for g in gpus}
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8 or f[0].lower() not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        hi = sorted(sm)[len(sm) // 4:]  # under load: drop the idle quartile
        return {"sm_mhz": statistics.median(hi), "sm_max_mhz": max(mx), "samples": len(sm),
                "power_w_max": max(power) if power else None, "reasons": sorted(reasons)}


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="cx", choices=["cx", "reference"])
    p.add_argument("--batch", type=int, default=2, help="prompts per prefill instance per step")
    p.add_argument("--min-len", type=int, default=512)
    p.add_argument("--max-len", type=int, default=8192)
    p.add_argument("--layers", type=int, default=32, help="model depth (32 = Llama-3-8B)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-mode", default="auto", choices=["auto", "push", "pull"],
                   help="layerwise KV transfer between GPUs: the prefill GPU pushes, or the decode GPU pulls "
                        "(auto: pull for N >= 2; one GPU always pushes into its local decode cache)")
    p.add_argument("--no-sub-metrics", action="store_true",
                   help="skip the EP layer and weight-sync measurements after the PD steps")
    args = p.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    sys.path.insert(0, ROOT)
    from connex_b200.bench.pd_bench import run_pd_bench
    res = run_pd_bench(args, ClockSampler, finalize=False)
    import torch
    import torch.distributed as dist
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if not args.no_sub_metrics:
        from connex_b200.bench.sub_metrics import run_sub_metrics
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        sub = run_sub_metrics(world, rank, dev, layers=args.layers)
        if world > 1:
            # serving under load: Poisson arrivals on every prefill/decode pair
            from datetime import timedelta
            from connex_b200.bench.pd_serving_bench import parser as serving_parser, run_serving
            torch.cuda.empty_cache()
            cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=300))
            sargs = serving_parser().parse_args(["--qps", "4", "--duration", "10", "--layers", str(args.layers),
                                                 "--min-len", str(args.min_len), "--max-len", str(args.max_len)])
            srv = run_serving(sargs, world, rank, int(os.environ.get("LOCAL_RANK", "0")), cpu)
            if sub is not None and srv is not None:
                sub.update({f"serving_{k}": srv[k] for k in ("qps_per_pair", "duration_s", "requests", "completed",
                                                               "ttft_p50_ms", "ttft_p99_ms", "tpot_p50_ms",
                                                               "output_tok_s")})
        if res is not None:
            res["sub_metrics"] = sub
    if world > 1 and dist.is_initialized():
        dist.destroy_process_group()
    if res is not None:
        res.update({"metric": METRIC, "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
                    "vs_baseline": round(res["value"] / PUBLISHED_KV_GBPS, 2) if res.get("value") else None,
                    "vs_baseline_note": ("cross-hardware: the published figure is a 1024-token prompt's KV over "
                                         "100 Gb InfiniBand between A40 nodes, not a B200 measurement")})
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

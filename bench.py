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
    ref = os.path.join(ROOT, "baseline", "_ref")
    reason = None
    if not os.path.isdir(os.path.join(ref, "connex")):
        reason = "reference not installed under baseline/_ref"
    else:
        # Probe the reference's stock PD data-plane selection in a clean interpreter
        # (our own `connex` package must not shadow it).
        code = ("import sys; sys.path.insert(0, %r); import importlib.util as u;"
                "print('connex_rs' if u.find_spec('connex_rs') else '',"
                " 'mooncake' if u.find_spec('mooncake') else '')") % ref
        out = subprocess.run([sys.executable, "-I", "-c", code], capture_output=True, text=True,
                             cwd="/", timeout=120).stdout.strip()
        if not out:
            reason = ("reference PD KV data plane needs connex-rs (empty git submodule, no Rust "
                      "toolchain) or Mooncake/UCX (not installed); its stock path cannot move GPU KV offline")
    if reason is not None:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
        return
    raise SystemExit("reference data plane present but no driver for it is implemented")


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

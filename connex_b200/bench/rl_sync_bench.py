"""RL elastic weight-sync scenario on one box: a Llama-3-8B trainer sharded
FSDP-style (dim-0 shards, fp32 master) on ranks 0-1 (``--trainers``) pushes
every round into the bf16 engine-layout weight arenas of the rollout replicas
on the other ranks
(q|k|v and gate/up fused by the broadcast kernel); weights are perturbed
before every round.  One rollout replica leaves in the middle of a round and
a standby replica joins in the middle of a later one.

Per round the line reports the device time from a common barrier to the last
consuming replica holding the new version (CUDA events, max over ranks).
The leaving replica stops waiting mid-round and nobody waits for it; the
joiner attaches once its copy is current: in multicast mode the NVSwitch has
been delivering every round to its bound arena (warm standby, attach = check
its flag), in p2p mode it reads a member's arena over NVLink
(``WeightBroadcast.catch_up``).  Every consuming replica checks an int64
checksum of its arena against the trainers' checksum of the same bytes.

    torchrun --nproc-per-node 4 -m connex_b200.bench.rl_sync_bench --rounds 10
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
from datetime import timedelta
from typing import Dict, List

import torch
import torch.distributed as dist

from connex_b200.models.llama import LlamaConfig, random_trainer_weights
from connex_b200.parallel.wsync import WeightBroadcast, apply_local, engine_manifest, plan_jobs, shard_dim0

def _checksum(arena_bytes: torch.Tensor) -> int:
    return int(arena_bytes.view(torch.int32).sum(dtype=torch.int64).item())


def run(cfg: LlamaConfig, rounds: int = 10, mode: str = "auto", leave_round: int = 3, join_round: int = 5,
        verify: bool = True, trainers: int = 2) -> Dict:
    world, rank = dist.get_world_size(), dist.get_rank()
    TRAINERS = tuple(range(trainers))
    if world < trainers + 1:
        raise SystemExit(f"the RL sync scenario needs {trainers} trainer rank(s) and at least one rollout rank")
    dev = torch.device("cuda", torch.cuda.current_device())
    rollouts = list(range(len(TRAINERS), world))
    standby = rollouts[-1]                      # joins at join_round
    leaver = rollouts[-2] if len(rollouts) > 2 else rollouts[-1]
    if leaver == standby:                       # two rollouts: the leaver comes back as the joiner
        members = list(rollouts)
    else:
        members = rollouts[:-1]
    m = engine_manifest(cfg)
    local = starts = None
    if rank in TRAINERS:
        full = random_trainer_weights(cfg, dev, dtype=torch.float32, seed=0)
        local, starts = shard_dim0(full, TRAINERS.index(rank), len(TRAINERS))
        local = {k: v.clone() for k, v in local.items()}
        del full
        torch.cuda.empty_cache()
    bc = WeightBroadcast(cfg, mode=mode, srcs=list(TRAINERS), timeout_s=30.0)
    scratch = torch.empty(m.total, dtype=torch.uint8, device=dev) if (verify and rank in TRAINERS) else None
    n_tasks = None
    per_round: List[float] = []
    events: Dict[str, float] = {}
    checks = 0
    stale_joiner = False
    for r in range(rounds):
        if rank in TRAINERS:
            with torch.no_grad():
                for t in local.values():
                    t.add_(1e-3)                # this round's update
        consuming = list(members)
        wait = True
        if r == leave_round and rank == leaver:
            wait = False                        # leaves mid-round: stops consuming
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        bc.sync(local, n_tasks, starts, members=consuming, wait=wait)
        b.record()
        torch.cuda.synchronize()
        bc.check()
        if n_tasks is None:
            box = [None] * world
            dist.all_gather_object(box, bc._jobs[2] if bc.is_src else None)
            n_tasks = [box[t] for t in TRAINERS]
        ms = a.elapsed_time(b) if (rank in TRAINERS or (rank in consuming and wait)) else 0.0
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        per_round.append(float(t.item()))
        if r == leave_round:
            members = [x for x in members if x != leaver]
            events["leave_round_ms"] = per_round[-1]
        if r == join_round:
            torch.cuda.synchronize()
            dist.barrier()
            j0, j1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            j0.record()
            source = next((x for x in members if x != standby), None)
            stale_joiner = not bc.mc and source is None     # nobody to copy from: the next round fills it
            if rank == standby and not bc.mc and source is not None:
                bc.catch_up(source)             # read a member's arena over NVLink
            elif rank == standby and bc.mc:
                from connex_b200 import ops    # warm standby: the multicast rounds are all there
                ops.wait_flag(bc.flag_addr, bc.received & 0xFFFFFFFF, bc.status, 5.0)
            j1.record()
            torch.cuda.synchronize()
            bc.check()
            t = torch.tensor([j0.elapsed_time(j1) if rank == standby else 0.0], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            events["join_catch_up_ms"] = None if stale_joiner else float(t.item())
            events["join_round_ms"] = per_round[-1]
            if standby not in members:
                members = members + [standby]
        if verify and (r in (0, leave_round, join_round, rounds - 1)):
            if rank in TRAINERS:
                scratch.zero_()
                apply_local(bc._jobs[0], scratch)
                torch.cuda.synchronize()
                mine = _checksum(scratch)
            else:
                mine = None
            box = [None] * world
            dist.all_gather_object(box, mine)
            want = sum(box[t] for t in TRAINERS)
            skip = rank not in members or (r == join_round and stale_joiner and rank == standby)
            ok = torch.tensor([1 if (skip or _checksum(bc.arena[:m.total]) == want) else 0],
                              dtype=torch.int32, device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok.item()) != 1:
                raise RuntimeError(f"round {r}: a member's arena does not match the trainers' bytes")
            checks += 1
    bc.close()
    steady = [x for i, x in enumerate(per_round) if i not in (0, leave_round, join_round)]
    return {"mode": "multicast" if bc.mc else "p2p", "rounds": rounds, "trainers": len(TRAINERS),
            "rollouts_start": len(rollouts) - (0 if leaver == standby else 1), "engine_bytes": m.total,
            "round_ms": [round(x, 3) for x in per_round], "median_round_ms": round(statistics.median(steady), 3),
            **{k: (None if v is None else round(v, 3)) for k, v in events.items()}, "verified_rounds": checks}


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--rounds", type=int, default=10)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--modes", default="multicast,p2p")
    p.add_argument("--no-verify", action="store_true")
    p.add_argument("--trainers", type=int, default=2, help="FSDP trainer ranks (the first ones)")
    a = p.parse_args()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
    cfg = LlamaConfig(layers=a.layers)
    out = {}
    for mode in a.modes.split(","):
        try:
            out[mode] = run(cfg, a.rounds, mode, verify=not a.no_verify, trainers=a.trainers)
        except RuntimeError as ex:
            if "multicast is not available" not in str(ex):
                raise
            out[mode] = {"unavailable": str(ex)}
        torch.cuda.empty_cache()
    if dist.get_rank() == 0:
        print(json.dumps({"bench": "rl_sync", "model": f"Llama-3-8B architecture ({a.layers} layers)",
                          "n_gpus": dist.get_world_size(), "results": out}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""RL weight-sync benchmark: Llama-3-8B trainer fp32 master weights ->
bf16 engine weights (fused q|k|v, interleaved gate/up) on every other GPU
of one box.

Arms (all end with the engine-layout bf16 weights in every receiver's live
weight arena):

* ``fused_mc``  -- :class:`WeightBroadcast` over NVLink multicast (one
  kernel reads fp32, casts, re-lays out and stores through the multicast
  address; receivers wait on a device flag);
* ``fused_relay`` -- the same kernel scattering each round of pieces to the
  receiver that owns their arena slice; each receiver multicasts its share
  of the round on to every arena as soon as it lands;
* ``fused_p2p`` -- the same kernel storing to each receiver's peer address;
* ``nccl``      -- conventional: PyTorch cast + cat + interleave on the
  trainer into a bf16 staging arena, then ``dist.broadcast`` (NCCL).

N = 1 times the local fused conversion only (``local``).  Device time by
CUDA events from a common barrier, max over ranks; weights (32 GB fp32,
16 GB bf16) exceed L2.
"""
from __future__ import annotations

import json
import os
from datetime import timedelta
from typing import Dict

import torch
import torch.distributed as dist

from connex_b200.models.llama import LlamaConfig, random_trainer_weights
from connex_b200.parallel.wsync import WeightBroadcast, apply_local, engine_manifest, fuse_reference, plan_jobs


def _ev():
    return torch.cuda.Event(enable_timing=True)


def _max(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time(fn, iters: int, world: int) -> float:
    ms = []
    for _ in range(iters):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = _ev(), _ev()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ms.append(_max(a.elapsed_time(b), world))
    return sorted(ms)[len(ms) // 2]


def run(cfg: LlamaConfig, iters: int = 5, warmup: int = 3) -> Dict:
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    m = engine_manifest(cfg)
    named = random_trainer_weights(cfg, dev, dtype=torch.float32, seed=1) if rank == 0 else None
    out: Dict = {"engine_bytes": m.total, "receivers": max(world - 1, 1)}
    if world == 1:
        jobs, _, _ = plan_jobs(cfg, m, named)
        arena = torch.empty(m.total, dtype=torch.uint8, device=dev)
        for _ in range(warmup):
            apply_local(jobs, arena)
        out["local_ms"] = _time(lambda: apply_local(jobs, arena), iters, 1)
        return out
    for mode in ("multicast", "relay", "relay_p2p", "p2p"):
        try:
            bc = WeightBroadcast(cfg, mode=mode)
        except RuntimeError as e:
            out[f"fused_{mode}_ms"] = None
            out[f"fused_{mode}_error"] = str(e)[:120]
            continue
        n_tasks = plan_jobs(cfg, m, named)[1] if rank == 0 else None
        box = [n_tasks]
        dist.broadcast_object_list(box, src=0)
        n_tasks = box[0]
        for _ in range(warmup):
            bc.sync(named, n_tasks)
        out[f"fused_{mode}_ms"] = _time(lambda: bc.sync(named, n_tasks), iters, world)
        torch.cuda.synchronize()
        bc.check()
        bc.close()
        del bc
        torch.cuda.empty_cache()
    staging = torch.empty(m.total, dtype=torch.uint8, device=dev)

    def nccl():
        if rank == 0:
            fused = fuse_reference(cfg, named)
            for e in m.entries:
                staging[e.offset:e.offset + e.nbytes].copy_(fused[e.name].view(-1).view(torch.uint8))
            del fused
        dist.broadcast(staging, src=0)
    for _ in range(warmup):
        nccl()
    out["nccl_ms"] = _time(nccl, iters, world)
    return out


def unpack_jobs(jobs: torch.Tensor, packed: torch.Tensor, arena: torch.Tensor) -> None:
    """Scatter a packed bf16 buffer (the job sources one after another, each
    ``rows x cols``) into the engine arena at the jobs' destination rows, with
    PyTorch strided copies (the NCCL baseline's receive side)."""
    a16 = arena.view(torch.bfloat16)
    off = 0
    for _, doff, rows, cols, _, dld, blk, bstride, boff, _, _, _ in jobs.tolist():
        n = rows * cols
        seg = packed[off:off + n]
        off += n
        nblk = rows // blk
        dst = a16.as_strided((nblk, blk, cols), (bstride * dld if nblk > 1 else dld * blk, dld, 1),
                             doff // 2 + boff * dld)
        dst.copy_(seg.view(nblk, blk, cols))


def run_sharded(cfg: LlamaConfig, trainers: int = 2, iters: int = 3, warmup: int = 2) -> Dict:
    """Trainer sharded FSDP-style (dim-0 shards, fp32) on ranks ``0..trainers-1``
    -> bf16 engine arenas on the other ranks.  Arms: the fused broadcast with
    every shard as a multicast source, and NCCL: each trainer casts its shard
    with PyTorch into a packed bf16 buffer and broadcasts it, every receiver
    scatters it into the engine layout with PyTorch copies."""
    from connex_b200.parallel.wsync import shard_dim0
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    m = engine_manifest(cfg)
    srcs = list(range(trainers))
    local = starts = None
    if rank in srcs:
        full = random_trainer_weights(cfg, dev, dtype=torch.float32, seed=1)
        local, starts = shard_dim0(full, rank, trainers)
        local = {k: v.clone() for k, v in local.items()}
        del full
        torch.cuda.empty_cache()
    jobs_cpu = plan_jobs(cfg, m, local, starts=starts)[0] if local is not None else None
    tables = [None] * world
    dist.all_gather_object(tables, (jobs_cpu.tolist(), int(sum(t.numel() for t in local.values())))
                           if jobs_cpu is not None else None)
    out: Dict = {"engine_bytes": m.total, "trainers": trainers, "receivers": world - trainers}
    try:
        bc = WeightBroadcast(cfg, mode="multicast", srcs=srcs)
        n_tasks = None
        bc.sync(local, n_tasks, starts)
        box = [None] * world
        dist.all_gather_object(box, bc._jobs[2] if bc.is_src else None)
        n_tasks = [box[t] for t in srcs]
        for _ in range(warmup):
            bc.sync(local, n_tasks, starts)
        out["fused_multicast_ms"] = _time(lambda: bc.sync(local, n_tasks, starts), iters, world)
        torch.cuda.synchronize()
        bc.check()
        bc.close()
        del bc
    except RuntimeError as e:
        out["fused_multicast_ms"] = None
        out["fused_multicast_error"] = str(e)[:120]
    torch.cuda.empty_cache()
    arena = torch.empty(m.total, dtype=torch.uint8, device=dev) if rank not in srcs else None
    bufs = {t: torch.empty(tables[t][1], dtype=torch.bfloat16, device=dev) for t in srcs if t != rank}
    jobs_of = {t: torch.tensor(tables[t][0], dtype=torch.int64) for t in srcs}

    def nccl():
        for t in srcs:
            if rank == t:
                buf = torch.cat([v.to(torch.bfloat16).reshape(-1) for v in local.values()])
            else:
                buf = bufs[t]
            dist.broadcast(buf, src=t)
            if arena is not None:
                unpack_jobs(jobs_of[t], buf, arena)
    for _ in range(warmup):
        nccl()
    out["nccl_ms"] = _time(nccl, iters, world)
    return out


def probe(cfg: LlamaConfig, iters: int = 3, warmup: int = 2) -> Dict:
    """Where a broadcast's time goes at this N (bf16 engine-layout source, so
    no cast): ``mc_copy`` multicast from rank 0 to everyone; ``scatter``
    rank 0 unicasts slice j of the arena to receiver j only (the sender's
    egress is the model once); ``fwd_mc`` / ``fwd_p2p`` every receiver sends
    its slice to all others through the multicast address / with unicast
    peer stores (the all-gather half).  Device time, max over ranks."""
    from connex_b200 import ops
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    m = engine_manifest(cfg)
    bc = WeightBroadcast(cfg, mode="multicast")
    total = m.total
    recv = list(range(1, world))
    R = len(recv)
    sl = -(-total // (R * 16)) * 16                    # slice bytes (16-byte aligned)
    named = {e.name: torch.randn(e.shape, device=dev).to(torch.bfloat16) for e in m.entries} if rank == 0 else None
    out: Dict = {"engine_bytes": total, "receivers": R, "slice_bytes": sl}
    n_tasks = [plan_jobs(cfg, m, named)[1] if rank == 0 else None]
    dist.broadcast_object_list(n_tasks, src=0)
    for _ in range(warmup):
        bc.sync(named, n_tasks[0])
    out["mc_copy_ms"] = _time(lambda: bc.sync(named, n_tasks[0]), iters, world)
    torch.cuda.synchronize()
    bc.check()
    jobs = plan_jobs(cfg, m, named)[0] if rank == 0 else None
    jobs_dev = jobs.to(dev) if jobs is not None else None
    state = {"target": bc.received}

    def scatter():
        dist.barrier()
        ctas = 0
        if rank == 0:
            ctas = ops._C.wsync(jobs_dev, jobs, total, [bc.peers[r] for r in recv],
                                [bc.peers[r] + total for r in recv], 0, 0, 0, sl)
        box = torch.tensor([ctas], device=dev)
        dist.broadcast(box, src=0)
        state["target"] += int(box.item())
        if rank != 0:
            ops.wait_flag(bc.flag_addr, state["target"] & 0xFFFFFFFF, bc.status, 10.0)
    for _ in range(warmup):
        scatter()
    out["scatter_ms"] = _time(scatter, iters, world)

    def my_slice_jobs():
        j = recv.index(rank)
        a, b = j * sl, min(total, (j + 1) * sl)
        cols = 4096                                    # 8 KB rows; the tail row separately
        full = (b - a) // (2 * cols)
        rows_ = []
        if full:
            rows_.append([bc.arena.data_ptr() + a, a, full, cols, cols, cols, full, 0, 0, 0, 0, full])
        tail = (b - a) - full * 2 * cols
        if tail:
            t0 = a + full * 2 * cols
            rows_.append([bc.arena.data_ptr() + t0, t0, 1, tail // 2, tail // 2, tail // 2, 1, 0, 0, 0,
                          1 if full else 0, 1])
        for r_ in rows_:                               # one task per 64 KB of output
            r_[11] = max(1, min(r_[2], (64 << 10) // (2 * r_[3])))
        t = 0
        for r_ in rows_:
            r_[10] = t
            t += -(-r_[2] // r_[11])
        return torch.tensor(rows_, dtype=torch.int64)
    if rank != 0:
        sj = my_slice_jobs()
        sj_dev = sj.to(dev)
        j = recv.index(rank)
        a, b = j * sl, min(total, (j + 1) * sl)
        segs = torch.tensor([[bc.arena.data_ptr() + a, bc.peers[r] + a, b - a] for r in recv if r != rank],
                            dtype=torch.int64, device=dev)

    def fwd_mc():
        dist.barrier()
        if rank != 0:
            ops._C.wsync(sj_dev, sj, total, [], [], bc.mc, 0, 0, 0)
    def fwd_p2p():
        dist.barrier()
        if rank != 0 and segs.shape[0]:
            ops.copy_segments(segs, int(segs[:, 2].sum().item()), status=bc.status)
    for name, fn in (("fwd_mc_ms", fwd_mc), ("fwd_p2p_ms", fwd_p2p)):
        if name == "fwd_mc_ms" and not bc.mc:
            continue
        for _ in range(warmup):
            fn()
        out[name] = _time(fn, iters, world)
    torch.cuda.synchronize()
    bc.check()
    bc.close()
    return out


def relay_timeline(cfg: LlamaConfig, warmup: int = 2, mode: str = "relay") -> Dict:
    """One relay broadcast with per-round events on every rank: when the
    trainer's round kernels end, and when each receiver saw a round land and
    finished forwarding it (ms from each rank's own start after the opening
    barrier).  Rank 0 gets the trainer's list and, per round, the earliest
    and latest receiver times."""
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    m = engine_manifest(cfg)
    named = random_trainer_weights(cfg, dev, dtype=torch.float32, seed=1) if rank == 0 else None
    bc = WeightBroadcast(cfg, mode=mode)
    n_tasks = plan_jobs(cfg, m, named)[1] if rank == 0 else None
    box = [n_tasks]
    dist.broadcast_object_list(box, src=0)
    for _ in range(warmup):
        bc.sync(named, box[0])
    torch.cuda.synchronize()
    bc.timeline = []
    bc.sync(named, box[0])
    torch.cuda.synchronize()
    bc.check()
    mine = bc.timeline[-1] if bc.timeline else {}
    allt = [None] * world
    dist.all_gather_object(allt, mine)
    bc.close()
    if rank != 0:
        return {}
    recv = [t for r, t in enumerate(allt) if r != 0]
    rounds = sorted({int(k[6:]) for t in recv for k in t if k.startswith("landed")})
    out = {"scatter_end_ms": [allt[0].get(f"scatter{r}") for r in rounds]}
    for tag in ("landed", "forwarded"):
        out[f"{tag}_ms_min_max"] = [(min(t[f"{tag}{r}"] for t in recv), max(t[f"{tag}{r}"] for t in recv))
                                    for r in rounds]
    return out


def main() -> None:
    import argparse
    p = argparse.ArgumentParser()
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--probe", action="store_true", help="time multicast / scatter / all-gather halves instead")
    p.add_argument("--relay-timeline", action="store_true", help="per-round events of one relay broadcast")
    p.add_argument("--relay-mode", default="relay", choices=["relay", "relay_p2p"])
    a = p.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    cfg = LlamaConfig(layers=a.layers)
    if a.relay_timeline:
        res = relay_timeline(cfg, mode=a.relay_mode)
        if dist.get_rank() == 0:
            print(json.dumps({"relay_timeline": res, "n_gpus": world}), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return
    if a.probe:
        res = probe(cfg, a.iters)
        if dist.get_rank() == 0:
            print(json.dumps({"wsync_probe": res, "n_gpus": world}), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return
    res = run(cfg, a.iters)
    if (dist.get_rank() if world > 1 else 0) == 0:
        gb = res["engine_bytes"] / 1e9
        for k in [k for k in list(res) if k.endswith("_ms") and res[k]]:
            res[k.replace("_ms", "_GBps_per_receiver")] = round(gb / (res[k] / 1e3), 1)
        print(json.dumps({"wsync": res, "n_gpus": world, "model": "llama3-8b", "src_dtype": "fp32"}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

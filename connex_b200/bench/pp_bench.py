"""Elastic pipeline-parallel benchmark: Llama-3-8B architecture (bf16,
random init) in 2 stages of 16 layers, R replicas per stage (N = 2R GPUs,
one process each), activations ``[batch, 4096]`` bf16 between stages over
elastic NCCL pair links, membership and failover through the directory.

Timeline (per stage-0 replica: ``--batch`` requests of ``--prompt`` random
token ids, then ``--steps`` greedy decode steps):

1. prefill through the pipeline, decode with K=1 steps;
2. at decode step ``--kill-at`` stage-1 replica 1 dies between steps (it
   takes the step, deregisters and closes without answering): its stage-0
   peer fails over to another stage-1 replica, which lacks the KV of those
   requests, so they come back as ``cx_missing`` and are prefilled again;
3. the killed replica rejoins ``--rejoin-after`` s later under the same
   identity at a new address (address migration, empty cache);
4. at step ``--kill2-at`` stage-1 replica 0 dies: every chain now fails over
   to the rejoined replica.

Reported (rank 0): decode tokens/s over the steady steps (device time of the
stage-0 step loops, max over stage-0 ranks), and each handover time = kill
-> first step with valid tokens for every request, measured on the host
clock of the one box (the event spans processes).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from connex.directory import DirectoryClient
from connex.pp.endpoint import PipelineEndpoint
from connex.pp.handover import CX_CTX, REQUEST_IDS
from connex.pp.link import Stage0Link, StageWorker
from connex.pp.membership import DirectoryMembership
from connex_b200.models.llama import LlamaConfig
from connex_b200.parallel.pplink import PairLinks
from connex_b200.runtime.pp import StageRuntime

MODEL = "llama3-8b-pp"


DATA_PLANE = {"links": "nccl"}


def _make_endpoint(stage, replica, dev, store, dir_addr, port=0):
    ep = PipelineEndpoint(MODEL, stage, 2, replica, data="link", links=None, device=str(dev), recv_timeout_s=30.0,
                          port=port)
    if DATA_PLANE["links"] == "chan":
        from connex_b200.parallel.p2pchan import ChanLinks
        ep.links = ChanLinks(dist.PrefixStore("ppchan/", store), ep.link_id, dev, slots=2, slot_bytes=256 << 20)
    else:
        ep.links = PairLinks(dist.PrefixStore("pplinks/", store), ep.link_id, dev, timeout_s=60)
    client = DirectoryClient(dir_addr, MODEL, stage, replica_idx=replica, local_addresses=[ep.address])
    client.start()
    client.start_event_listener()
    ep.attach_membership(DirectoryMembership(client, 2))
    client.register([ep.address])
    client.start_heartbeat(0.2)
    return ep, client


def _cfg(args) -> LlamaConfig:
    return LlamaConfig.tiny(layers=2) if args.tiny else LlamaConfig(layers=32)


def stage1_main(args, rank, replica, dev, store, dir_addr, n_s0):
    cfg = _cfg(args)
    half = cfg.layers // 2
    rt = StageRuntime(cfg, half, cfg.layers, dev, num_blocks=n_s0 * args.batch * (args.prompt + args.steps + 16) // 16 + 64,
                      max_tokens=args.batch * (args.prompt + args.steps), max_batch=args.batch,
                      max_ctx=args.prompt + args.steps + 16, seed=0)
    ep, client = _make_endpoint(1, replica, dev, store, dir_addr)
    store.set(f"ready/{rank}", "1")
    decode_seen = 0
    worker = StageWorker(ep, rt, rt.compute)
    lives = 0
    while True:
        if int(store.add("s0_done", 0)) >= n_s0:
            break
        td, ctx = ep.recv_forward(timeout_s=0.2)
        if td is None:
            continue
        if td.get("kind") == "decode":
            decode_seen += 1
        if replica == 1:
            die = lives == 0 and decode_seen == args.kill_at
        elif replica == 0:      # only once the first victim is back, so a chain is left to fail over to
            die = lives == 0 and decode_seen >= args.kill2_at and _has(store, "rejoin_t/1")
        else:
            die = False
        if die:
            # die between steps: the step was received (its transfer finished), it is never answered
            torch.cuda.synchronize(dev)
            store.set(f"kill_t/{replica}", repr(time.time()))
            client.deregister()
            client.stop()
            ep.close()
            ep.links.close()
            lives += 1
            if replica != 1:
                store.add("s1_exit", 1)
                return
            time.sleep(args.rejoin_after)
            rt.tables, rt.held = {}, {}           # back with an empty cache (same weights)
            rt.cache._free = list(range(rt.cache.num_blocks - 1, -1, -1))
            ep, client = _make_endpoint(1, replica, dev, store, dir_addr)   # new port: migrated address
            store.set(f"rejoin_t/{replica}", repr(time.time()))
            worker = StageWorker(ep, rt, rt.compute)
            continue
        worker.serve(td, ctx)
    client.deregister()
    client.stop()
    ep.close()
    ep.links.close()
    store.add("s1_exit", 1)


class _Stage0Hooks:
    def __init__(self):
        self.reprefill_rids = []

    def kv_held(self, rid):
        return 0

    def release(self, rids):
        pass

    def reprefill(self, rids):
        self.reprefill_rids = list(rids)

    def abort(self, rids):
        pass


def stage0_main(args, rank, replica, dev, store, dir_addr):
    cfg = _cfg(args)
    B, P, S = args.batch, args.prompt, args.steps
    rt = StageRuntime(cfg, 0, cfg.layers // 2, dev, num_blocks=B * (P + S + 16) // 16 + 64, max_tokens=B * (P + S),
                      max_batch=B, max_ctx=P + S + 16, seed=0)
    if args.replay:
        rt.enable_activation_log(B)
    ep, client = _make_endpoint(0, replica, dev, store, dir_addr)
    warmed = ep.warm_stage(1)          # every stage-1 replica's links are set up before traffic
    ep.auto_warm = True                # and a replica that (re)joins gets warmed in the background
    hooks = _Stage0Hooks()
    link = Stage0Link(ep, hooks, recv_timeout_s=30.0)
    g = torch.Generator().manual_seed(1234 + replica)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=g)
    rids = [f"c{replica}-r{i}" for i in range(B)]
    gen = [[] for _ in range(B)]

    def pipeline_step(kind, ids_list, ctx, n_new, rows_rids):
        ids = torch.tensor(ids_list, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        td = {"kind": kind, REQUEST_IDS: rows_rids, CX_CTX: ctx, "n_new": n_new, "ids": ids}
        x = rt.compute(td, [])["x"]
        hooks.reprefill_rids = []
        out = link.step({"x": x, "kind": kind, "n_new": n_new}, request_ids=rows_rids, num_computed=ctx)
        return out["next"], list(hooks.reprefill_rids)

    def prefill(idx):
        toks = [prompts[i].tolist() + gen[i] for i in idx]
        nxt, again = pipeline_step("prefill", sum(toks, []), [0] * len(idx), [len(t) for t in toks],
                                   [rids[i] for i in idx])
        return nxt.tolist()

    nxt = prefill(list(range(B)))
    for i in range(B):
        gen[i].append(nxt[i])
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(S + 1)]
    handovers = []
    ev[0].record()
    for s in range(S):
        before = ep.current
        ctx = [P + len(gen[i]) - 1 for i in range(B)]
        nxt, again = pipeline_step("decode", [gen[i][-1] for i in range(B)], ctx, [1] * B, rids)
        nxt = nxt.tolist()
        if again:
            idx = [rids.index(r) for r in again]
            if args.replay:            # stage 0 still holds its part: replay its logged outputs
                x, lens = rt.replay([rids[i] for i in idx])
                hooks.reprefill_rids = []
                out = link.step({"x": x, "kind": "prefill", "n_new": lens}, request_ids=[rids[i] for i in idx],
                                num_computed=[0] * len(idx))
                fixed = out["next"].tolist()
            else:
                fixed = prefill(idx)   # prompt + generated so far: its last position is this step's token
            for j, i in enumerate(idx):
                nxt[i] = fixed[j]
            t_ok = time.time()
            if before is not None and _has(store, f"kill_t/{before}"):
                kt = float(store.get(f"kill_t/{before}").decode())
                handovers.append({"dead_replica": before, "to_replica": ep.current,
                                  "ms": round((t_ok - kt) * 1e3, 2), "reprefilled": len(again), "step": s})
        for i in range(B):
            gen[i].append(nxt[i])
        ev[s + 1].record()
    torch.cuda.synchronize(dev)
    dev_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(S)]
    store.add("s0_done", 1)
    client.deregister()
    client.stop()
    ep.close()
    ep.links.close()
    return {"rank": rank, "dev_ms": dev_ms, "handovers": handovers, "stats": dict(link.stats),
            "failovers": ep.stats.get("failovers", 0)}


def _has(store, key) -> bool:
    """Non-blocking existence check (a timed-out ``wait`` costs a socket poll)."""
    return bool(store.check([key]))


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--prompt", type=int, default=1024)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--kill-at", type=int, default=100)
    p.add_argument("--kill2-at", type=int, default=180)
    p.add_argument("--rejoin-after", type=float, default=1.0)
    p.add_argument("--tiny", action="store_true", help="small model of the same geometry (smoke run)")
    p.add_argument("--no-replay", dest="replay", action="store_false",
                   help="after a failover, recompute stage 0 instead of replaying its logged outputs")
    p.add_argument("--links", choices=["nccl", "chan"], default="nccl",
                   help="activation data plane: NCCL pair groups, or GPU-driven NVLink channels")
    a = p.parse_args()
    DATA_PLANE["links"] = a.links
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    store = dist.distributed_c10d._get_default_store()
    n_s0 = world // 2
    dport = int(os.environ["MASTER_PORT"]) + 17
    dir_addr = f"127.0.0.1:{dport}"
    server = None
    if rank == 0:
        from connex.directory_server import DirectoryServer
        server = DirectoryServer(dir_addr, lease_s=2.0)
        server.start()
    dist.barrier()
    res = None
    if rank < n_s0:
        # wait until every stage-1 replica is up before routing
        for r in range(n_s0, world):
            store.wait([f"ready/{r}"], timedelta(seconds=600))
        res = stage0_main(a, rank, rank, dev, store, dir_addr)
    else:
        stage1_main(a, rank, rank - n_s0, dev, store, dir_addr, n_s0)
    allr = [None] * world
    dist.all_gather_object(allr, res)
    if rank == 0:
        s0 = [r for r in allr if r]
        steady = [statistics.median(r["dev_ms"][5:a.kill_at - 2]) for r in s0]
        ms = max(steady)
        print(json.dumps({"pp": {"n_gpus": world, "links": a.links, "replay": a.replay, "stages": 2,
                                 "replicas_per_stage": n_s0,
                                 "batch": a.batch,
                                 "prompt": a.prompt, "decode_steps": a.steps, "step_ms_p50_max_over_ranks": ms,
                                 "decode_tok_s": round(n_s0 * a.batch / (ms / 1e3), 1),
                                 "handovers": [h for r in s0 for h in r["handovers"]],
                                 "failovers": [r["failovers"] for r in s0],
                                 "retries": [r["stats"].get("retries") for r in s0]}}), flush=True)
    dist.barrier()
    if server is not None:
        server.stop()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

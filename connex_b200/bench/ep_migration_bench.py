"""EP MoE serving with live expert migration and a rank failure:
Qwen3-30B-A3B-style MoE (48 layers, hidden 2048, 128 experts, top-8,
expert FFN 768, 32 q / 4 kv heads, bf16, random init), EP over N GPUs (one
process each, data-parallel attention), router logits N(0,1) + Zipf(1.2).

Timeline (each rank decodes ``--batch`` requests with ``--ctx`` tokens of
context per step):

1. steady decode;
2. at step ``--migrate-at`` the 16 experts of rank 3 are copied to spare
   slots of ranks 0-2 (all 48 layers, 7.2 GB) while decode continues: each
   receiver pulls its share over NVLink from rank 3's weight memory (CUDA IPC
   mapping) with this package's copy kernel on a low-priority stream, then the
   placement commits the new slots (two epochs: staged, then routable) at an
   agreed step boundary;
3. at step ``--fail-at`` rank 3 leaves between steps; the survivors learn it
   from the store before their next launch, drop its slots from the placement
   and mark it dead in the EP layer (its peer-table column points at local
   sinks, wait targets count live ranks: no buffer or IPC mapping is rebuilt),
   and decode continues.

Reported (rank 0): decode step time before / during / after migration and
after the failure (device time, max over ranks), the migration copy time and
bandwidth (device time on the receivers, max), and the failure stall (rank 3
leaves -> first completed step of the rebuilt group, host clock of the box).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from datetime import timedelta
from typing import Dict, List

import torch
import torch.distributed as dist

from connex.ep.placement import Move, PlacementTable, l2p_tensors
from connex_b200 import ops
from connex_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeRank, expert_weights, zipf_bias, zipf_router
from connex_b200.parallel.ep import EPBuffers, EPConfig, EPMoE, map_remote, peer_table
from connex_b200.parallel.peer import PeerHandle, PeerMapper, export_tensor

VICTIM = 3


def _store_exchange(store, key: str, me: int, members: List[int], value) -> Dict[int, object]:
    import pickle
    store.set(f"{key}/{me}", pickle.dumps(value))
    out = {}
    for r in members:
        store.wait([f"{key}/{r}"], timedelta(seconds=300))
        out[r] = pickle.loads(store.get(f"{key}/{r}"))
    return out


class Group:
    """The EP group over ``members`` (global ranks) as seen by ``me``."""

    def __init__(self, key, store, me, members, cfg_ep: EPConfig, model: Qwen3MoeRank, dev):
        self.members = list(members)
        self.idx = self.members.index(me)
        self.bufs = EPBuffers(cfg_ep, dev)
        self.mapper = PeerMapper(dev.index)
        ex = _store_exchange(store, key, me, self.members, self.bufs.exports())
        addrs = [self.bufs.addresses() if r == me else map_remote(ex[r], self.mapper) for r in self.members]
        self.peers = peer_table(addrs, dev)
        self.moe = EPMoE(cfg_ep, self.idx, self.bufs, self.peers, model.w13[0], model.w2[0])
        model.moe = self.moe

    def close(self):
        self.mapper.close()


def l2p_for(table: PlacementTable, members: List[int], S: int, dev, layers: int, max_rep: int):
    """Per-layer l2p with physical slots renumbered to the group's rank order."""
    out = []
    view = table.view()
    for l in range(layers):
        a, c = l2p_tensors(view, l, "cpu", max_rep)
        a = a.clone()
        for e in range(a.shape[0]):
            for j in range(int(c[e])):
                p = int(a[e, j])
                r, loc = divmod(p, S)
                a[e, j] = members.index(r) * S + loc
        out.append((a.to(dev), c.to(dev)))
    return [x[0] for x in out], [x[1] for x in out]


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--ctx", type=int, default=1024)
    p.add_argument("--steps", type=int, default=60)
    p.add_argument("--migrate-at", type=int, default=15)
    p.add_argument("--fail-at", type=int, default=40)
    p.add_argument("--spare", type=int, default=8)
    p.add_argument("--copy-ctas", type=int, default=32)
    p.add_argument("--tiny", action="store_true")
    a = p.parse_args()
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=timedelta(seconds=900))
    store = dist.distributed_c10d._get_default_store()
    cfg = Qwen3MoeConfig.tiny() if a.tiny else Qwen3MoeConfig()
    E, L, N = cfg.experts, cfg.layers, world
    per = E // N
    S = per + max(a.spare, -(-per // 3))     # room for the victim's experts on 3 receivers
    victim = VICTIM if N > VICTIM else N - 1
    rows = [[(r * per + j) if j < per else -1 for r in range(N) for j in range(S)] for _ in range(L)]
    table = PlacementTable(E, N, S, rows)
    B, C = a.batch, a.ctx
    blocks_per = -(-(C + a.steps + 1) // cfg.block_size)
    model = Qwen3MoeRank(cfg, rank, S, rows, dev, num_blocks=B * blocks_per + 8, max_tokens=B)
    model.cache.kv.normal_(0, 1)           # a filled context (its values do not matter for timing)
    cfg_ep = EPConfig(N, S, cfg.hidden, cfg.moe_ffn, cfg.top_k, max_tokens=B)
    members = list(range(N))
    group = Group("ep0", store, rank, members, cfg_ep, model, dev)
    max_rep = 2
    l2p, cnt = l2p_for(table, members, S, dev, L, max_rep)
    # per-rank synthetic routing pool (cycled), request state
    gen = torch.Generator(device=dev)
    gen.manual_seed(100 + rank)
    bias = zipf_bias(cfg, 7, dev)
    pool = [[zipf_router(B, cfg, gen, bias) for _ in range(L)] for _ in range(4)]
    bt = torch.arange(B * blocks_per, dtype=torch.int32, device=dev).view(B, blocks_per)
    ws = ops.decode_workspace(B, cfg.heads, C + a.steps + 1, dev)
    ids = torch.randint(0, cfg.vocab_size, (B,), dtype=torch.int32, device=dev)
    # weight exports of the victim (receivers pull from them)
    wexp = _store_exchange(store, "w", rank, members, [export_tensor(model.w13).to_dict(),
                                                        export_tensor(model.w2).to_dict()])
    side = torch.cuda.Stream(dev, priority=0)
    moves: List[Move] = []
    receivers = [r for r in range(N) if r != victim][:3]
    ex = [e for e in range(E) if victim * per <= e < (victim + 1) * per]
    for i, e in enumerate(ex):
        r = receivers[i % len(receivers)]
        j = per + i // len(receivers)
        for l in range(L):
            moves.append(Move(l, e, r * S + j, victim * S + (e - victim * per)))
    mine = [m for m in moves if m.dst // S == rank]
    copy_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    copy_started = copied = committed = failed = False
    commit_at = fail_rebuild_ms = None
    t_ms: Dict[str, List[float]] = {"steady": [], "migrating": [], "after_commit": [], "after_failure": []}
    status = ops.new_status(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    first_after_fail = None
    for step in range(a.steps):
        if step == a.fail_at and not failed:
            # rank `victim` leaves between steps; everyone knows it before the next launch
            if rank == victim:
                torch.cuda.synchronize(dev)
                store.set("fail_t", repr(time.time()))
                group.close()
                break
            store.wait(["fail_t"], timedelta(seconds=300))
            table.mark_down(victim)
            table.commit()
            l2p, cnt = l2p_for(table, members, S, dev, L, max_rep)
            group.moe.mark_dead(victim)        # same buffers and mappings; its memory is never touched again
            failed = True
            first_after_fail = step
        if step == a.migrate_at and mine and not copy_started:
            mapper = PeerMapper(dev.index)
            src13 = mapper.open(PeerHandle.from_dict(wexp[victim][0]))
            src2 = mapper.open(PeerHandle.from_dict(wexp[victim][1]))
            e13 = 2 * cfg.moe_ffn * cfg.hidden * 2
            e2 = cfg.hidden * cfg.moe_ffn * 2
            segs = []
            for m in mine:
                js, jd = m.src % S, m.dst % S
                segs.append((src13 + (m.layer * S + js) * e13, model.w13.data_ptr() + (m.layer * S + jd) * e13, e13))
                segs.append((src2 + (m.layer * S + js) * e2, model.w2.data_ptr() + (m.layer * S + jd) * e2, e2))
            segs_t = torch.tensor(segs, dtype=torch.int64, device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                copy_ev[0].record(side)
                ops.copy_segments(segs_t, sum(s[2] for s in segs), max_ctas=a.copy_ctas, status=status)
                copy_ev[1].record(side)
            copy_started = True
        if step == a.migrate_at:
            table.begin_moves(moves)          # epoch 1: staged, not routable
            table.commit()
        if copy_started and not copied and copy_ev[1].query():
            copied = True
            store.add("copied", 1)
        if step > a.migrate_at and not committed and commit_at is None and rank == 0:
            if int(store.add("copied", 0)) >= len(receivers):
                store.set("commit_at", str(step + 2))
        if step > a.migrate_at and commit_at is None and store.check(["commit_at"]):
            commit_at = int(store.get("commit_at"))
        if commit_at is not None and step == commit_at and not committed:
            table.finish_moves(moves)          # epoch 2: the new slots are routable
            table.commit()
            l2p, cnt = l2p_for(table, members, S, dev, L, max_rep)
            committed = True
        routing = pool[step % len(pool)]
        ctx = C + step + 1
        pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
        slots = (bt[:, (ctx - 1) // cfg.block_size].long() * cfg.block_size + (ctx - 1) % cfg.block_size)
        lens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
        ev0.record()
        ids = model.decode(ids, pos, slots, bt, lens, ctx, ws, routing, l2p, cnt)
        ev1.record()
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1)
        if first_after_fail == step:
            fail_rebuild_ms = (time.time() - float(store.get("fail_t"))) * 1e3
        phase = ("after_failure" if failed else "after_commit" if committed else
                 "migrating" if step >= a.migrate_at else "steady")
        t_ms[phase].append(ms)
    torch.cuda.synchronize(dev)
    ops.check_status(status, "expert copy")
    ops.check_status(group.bufs.status, "ep")
    copy_ms = copy_ev[0].elapsed_time(copy_ev[1]) if copied else None
    # verify a few migrated expert slots against freshly drawn weights
    ok = True
    for m in mine[:: max(1, len(mine) // 4)]:
        w13, w2 = expert_weights(cfg, m.layer, m.expert, dev)
        ok &= bool(torch.equal(model.w13[m.layer, m.dst % S], w13) and torch.equal(model.w2[m.layer, m.dst % S], w2))
    res = {"rank": rank, "t": t_ms, "copy_ms": copy_ms, "copy_bytes": len(mine) * cfg.expert_bytes_per_layer,
           "fail_ms": fail_rebuild_ms, "verified": ok}
    allr = [None] * world
    dist.all_gather_object(allr, res)
    if rank == 0:
        def phase_max(k):
            v = [statistics.median(r["t"][k]) for r in allr if r["t"][k]]
            return round(max(v), 3) if v else None
        cps = [(r["copy_ms"], r["copy_bytes"]) for r in allr if r["copy_ms"]]
        print(json.dumps({"ep_migration": {
            "n_gpus": N, "model": "qwen3-30b-a3b-geometry" if not a.tiny else "tiny", "batch_per_rank": B,
            "ctx": C, "step_ms": {k: phase_max(k) for k in t_ms},
            "migrated_experts": len(ex), "migrated_bytes": sum(b for _, b in cps),
            "copy_ms_max": round(max(c for c, _ in cps), 3) if cps else None,
            "copy_GBps_per_receiver": [round(b / c / 1e6, 1) for c, b in cps],
            "failure_stall_ms_max": round(max(r["fail_ms"] for r in allr if r["fail_ms"]), 1)
            if any(r["fail_ms"] for r in allr) else None,
            "weights_verified": all(r["verified"] for r in allr)}}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""PD-disaggregated serving under Poisson load (Llama-3-8B architecture,
random-init bf16 weights, random token ids): prefill GPU ``p`` pushes each
batch's KV layer by layer into decode GPU ``p + N/2`` (the ``kv_push_layer``
kernel over the peer mapping, overlapped with the remaining prefill layers);
the decode GPU runs continuous batching until every request has its output
tokens.  The serving counterpart of the PD measurements the reference
publishes (TTFT / TPOT at a request rate, reference ``docs/results.md:289-296``).

Control between the two GPUs of a pair is a ZeroMQ PAIR socket:

* the prefill side owns the decode cache's block allocator (the decode side
  returns blocks with ``FREE`` when a request finishes), so a batch needs no
  round trip before its push;
* after a batch's prefill and pushes completed on the device, ``ARRIVE``
  carries the requests (arrival time, prompt length, decode blocks, first
  token) and the CTA count the decode side adds to its cumulative ready
  target; the decode side admits them between two decode steps after a
  bounded device wait on the ready counter.

Decode failure (``--kill-at S``): the prefill side keeps each request's
prompt KV as a lease until the decode side reports the request finished.
At ``S`` seconds the decode instance dies: its running and admitted requests
are lost and it says so (``DEAD``, what its peer learns from the engine's
peer-failure event); after ``--restart-s`` a replacement serves on the same
GPU (``READY``) and the prefill side refills it from the held KV (pushes
only, no prefill compute).  The lost requests decode again from their first
token; ``resume_stall`` is kill -> decoding again.  Nothing is killed on the
device: the instance's host state is dropped between two decode steps.

Reported (host wall clock; one host, so the clocks of the two processes
agree): TTFT = arrival -> request admitted on the decode GPU with its KV and
first token in place (queueing + prefill + KV push + admission); TPOT = mean
gap between its decode tokens; output tokens/s; and the device-timed push
bandwidth of the KV kernels.

    torchrun --nproc-per-node 2 -m connex_b200.bench.pd_serving_bench --qps 4 --duration 20
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from datetime import timedelta
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.distributed as dist
import zmq

from connex_b200 import ops
from connex_b200.models.llama import LlamaConfig, LlamaModel, LlamaWeights, PagedKVCache
from connex_b200.parallel.peer import PeerHandle, PeerMapper, export_tensor
from connex_b200.runtime.pd import (DecodeBatch, KVDestination, LayerwiseKVPusher, block_pairs,
                                    build_prefill_batch, decode_step)

PUSH_CTAS = 0   # one 128-thread CTA per SM (see LayerwiseKVPusher)


def arrivals(seed: int, pair: int, qps: float, duration: float, lo: int, hi: int, vocab: int):
    """Poisson arrivals in [0, duration): ``[(t, prompt)]``."""
    rng = np.random.default_rng([seed, pair, 7])
    out, t = [], 0.0
    while True:
        t += rng.exponential(1.0 / qps)
        if t >= duration:
            return out
        n = int(rng.integers(lo, hi + 1))
        out.append((t, rng.integers(0, vocab, size=n).tolist()))


def _pct(xs: List[float], q: float) -> float:
    return float(np.percentile(np.asarray(xs), q)) if xs else float("nan")


def prefill_side(args, cfg, weights, dev, sock, dst, n_dec_blocks: int) -> Dict:
    cache = PagedKVCache(cfg, args.prefill_blocks, dev)
    model = LlamaModel(weights, cache, max_tokens=args.token_budget, max_batch=args.max_running)
    pusher = LayerwiseKVPusher(cache, max_ctas=PUSH_CTAS)
    free = list(range(n_dec_blocks))                  # the decode cache's free blocks
    reqs = arrivals(args.seed, args.pair, args.qps, args.duration, args.min_len, args.max_len, cfg.vocab_size)
    need = [cache.blocks_needed(len(p) + args.out_tokens) for _, p in reqs]
    warm = build_prefill_batch(cache, [list(range(512))], dev)          # first-launch costs off the clock
    model.prefill(warm.ids, warm.positions, warm.slots, warm.seq_lens, warm.last_rows, warm.tile_info)
    torch.cuda.synchronize()
    cache.free(warm.src_blocks[0])
    t0 = time.time() + 0.5
    sock.send_pyobj({"op": "START", "t0": t0, "n": len(reqs)})
    queue: List[int] = []
    # KV leases: a request's prompt KV stays held on the prefill GPU until the
    # decode side reports it finished, so a decode that dies can be refilled
    held: Dict[int, dict] = {}
    lost: List[int] = []
    state = {"decode_up": True, "bye": False, "done": False, "repushed": 0}
    nxt_i, push_ms, push_bytes, batches = 0, 0.0, 0, 0

    def on_msg(m):
        if m["op"] == "FREE":
            for rid in m["rids"]:
                h = held.pop(rid)
                free.extend(h["dblocks"])
                cache.free(h["sblocks"])
        elif m["op"] == "DEAD":                         # the decode instance is gone
            state["decode_up"] = False
            for rid in m["lost"]:
                free.extend(held[rid]["dblocks"])      # the replacement starts with an empty cache
                lost.append(rid)
        elif m["op"] == "READY":                        # its replacement is serving
            state["decode_up"] = True
        elif m["op"] == "BYE":
            state["bye"] = True

    def drain(block_s: float = 0.0):
        if sock.poll(int(block_s * 1000)):
            while sock.poll(0):
                on_msg(sock.recv_pyobj())

    def take_blocks(n):
        b = free[:n]
        del free[:n]
        return b

    def send(ctas, rids, resumed=False):
        sock.send_pyobj({"op": "ARRIVE", "ctas": ctas, "resumed": resumed,
                         "reqs": [{"rid": i, "arrival": t0 + reqs[i][0], "len": len(reqs[i][1]),
                                   "blocks": held[i]["dblocks"], "first": held[i]["first"]} for i in rids]})

    while not state["bye"]:
        now = time.time()
        while nxt_i < len(reqs) and t0 + reqs[nxt_i][0] <= now:
            queue.append(nxt_i)
            nxt_i += 1
        drain()
        if lost and state["decode_up"] and sum(need[i] for i in lost) <= len(free):
            # refill the replacement from the held prompt KV: pushes only, no prefill compute
            rids, lost[:] = list(lost), []
            for i in rids:
                held[i]["dblocks"] = take_blocks(need[i])
            pairs = block_pairs([held[i]["sblocks"] for i in rids],
                                [held[i]["dblocks"][:len(held[i]["sblocks"])] for i in rids], dev)
            pusher.begin(pairs, dst, timing=True)
            for layer in range(cfg.layers):
                pusher.hook(layer)
            pusher.join()
            torch.cuda.synchronize()
            ops.check_status(pusher.status, "kv re-push")
            state["repushed"] += len(rids)
            send(pusher.launched, rids, resumed=True)
            continue
        if not queue or not state["decode_up"]:
            if nxt_i >= len(reqs) and not queue and not state["done"]:
                sock.send_pyobj({"op": "DONE"})        # no new requests; re-pushes may still follow
                state["done"] = True
            wait = 0.002 if nxt_i >= len(reqs) else max(0.0, min(0.002, t0 + reqs[nxt_i][0] - time.time()))
            drain(wait)
            continue
        pick, tokens, blocks = [], 0, 0
        for i in queue:
            n = len(reqs[i][1])
            if pick and tokens + n > args.token_budget:
                break
            if blocks + need[i] > len(free) or cache.free_blocks < cache.blocks_needed(tokens + n) + len(pick) + 1:
                break
            pick.append(i)
            tokens += n
            blocks += need[i]
        if not pick:
            drain(0.005)                              # wait for finished requests' blocks
            continue
        queue = queue[len(pick):]
        dblocks = [take_blocks(need[i]) for i in pick]
        batch = build_prefill_batch(cache, [reqs[i][1] for i in pick], dev)
        pairs = block_pairs(batch.src_blocks, [d[:len(s)] for d, s in zip(dblocks, batch.src_blocks)], dev)
        pusher.begin(pairs, dst, timing=True)
        first = model.prefill(batch.ids, batch.positions, batch.slots, batch.seq_lens, batch.last_rows,
                              batch.tile_info, layer_hook=pusher.hook)
        pusher.join()
        first_host = first[:len(pick)].cpu().tolist()       # synchronizes: prefill and pushes are done
        ops.check_status(pusher.status, "kv push")
        push_ms += pusher.push_ms()
        push_bytes += pusher.bytes
        batches += 1
        for i, d, sb, tok in zip(pick, dblocks, batch.src_blocks, first_host):
            held[i] = {"dblocks": d, "sblocks": sb, "first": tok}
        send(pusher.launched, pick)
    return {"requests": len(reqs), "batches": batches, "push_ms": push_ms, "push_bytes": push_bytes,
            "repushed": state["repushed"]}


def decode_side(args, cfg, weights, dev, sock, cache, ready) -> Dict:
    model = LlamaModel(weights, cache, max_tokens=args.max_running, max_batch=args.max_running)
    ws = ops.decode_workspace(args.max_running, cfg.heads, args.max_len + args.out_tokens + 2, dev)
    status = ops.new_status(dev)
    ids_host = torch.zeros(args.max_running, dtype=torch.int32).pin_memory()
    warm = DecodeBatch(cache, [[0]], [0], dev)                         # first-launch costs off the clock
    decode_step(model, warm, torch.zeros(1, dtype=torch.int32, device=dev), ws)
    torch.cuda.synchronize()
    start = sock.recv_pyobj()
    running: Dict[int, dict] = {}
    pending: List[dict] = []
    target, done, steps = 0, False, 0
    ttft, tpot, finished_tokens = [], [], 0
    t_first_token = t_last = None
    kill_at = start["t0"] + args.kill_at if args.kill_at > 0 else None
    t_kill, stalls, lost_n, n_done = None, [], 0, 0
    while True:
        while sock.poll(0 if (running or pending) else 2):
            m = sock.recv_pyobj()
            if m["op"] == "ARRIVE":
                target += m["ctas"]
                ops.wait_flag(ready.data_ptr(), target, status, timeout_s=30.0)   # bounded, stream-ordered
                for r in m["reqs"]:
                    r["resumed"] = m.get("resumed", False)
                pending.extend(m["reqs"])
            elif m["op"] == "DONE":
                done = True
        if kill_at is not None and time.time() >= kill_at:
            # this decode instance dies: its running and admitted requests are
            # lost; a replacement on the same GPU takes over after restart_s
            kill_at = None
            t_kill = time.time()
            lost = [r["rid"] for r in list(running.values()) + pending]
            lost_n = len(lost)
            running.clear()
            pending.clear()
            sock.send_pyobj({"op": "DEAD", "lost": lost})
            time.sleep(args.restart_s)
            sock.send_pyobj({"op": "READY"})
            continue
        while pending and len(running) < args.max_running:
            r = pending.pop(0)
            now = time.time()
            r.update(ctx=r["len"], last=r["first"], n_gen=1, t_admit=now)
            if r["resumed"]:
                stalls.append((now - t_kill) * 1e3)      # kill -> the request decodes again
            else:
                ttft.append((now - r["arrival"]) * 1e3)
            t_first_token = t_first_token or now
            running[r["rid"]] = r
        if not running:
            if done and not pending and (t_kill is None or len(stalls) >= lost_n):
                break
            continue
        rs = list(running.values())
        B = len(rs)
        batch = DecodeBatch(cache, [r["blocks"] for r in rs], [r["ctx"] for r in rs], dev)
        for j, r in enumerate(rs):
            ids_host[j] = r["last"]
        ids = ids_host[:B].to(dev, non_blocking=True)
        tok = decode_step(model, batch, ids, ws)[:B].cpu().tolist()
        steps += 1
        now = time.time()
        freed = []
        for r, t in zip(rs, tok):
            r["ctx"] += 1
            r["last"] = t
            r["n_gen"] += 1
            if r["n_gen"] >= args.out_tokens:
                if not r["resumed"]:
                    tpot.append((now - r["t_admit"]) * 1e3 / max(1, args.out_tokens - 1))
                finished_tokens += args.out_tokens
                n_done += 1
                freed.append(r["rid"])
                del running[r["rid"]]
        if freed:
            sock.send_pyobj({"op": "FREE", "rids": freed})
        t_last = now
    sock.send_pyobj({"op": "BYE"})
    ops.check_status(status, "decode ready wait")
    span = (t_last - start["t0"]) if t_last else float("nan")
    return {"ttft_ms": ttft, "tpot_ms": tpot, "decode_steps": steps, "output_tokens": finished_tokens,
            "span_s": span, "completed": n_done, "lost": lost_n, "stall_ms": stalls}


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser()
    p.add_argument("--qps", type=float, default=4.0)
    p.add_argument("--duration", type=float, default=20.0)
    p.add_argument("--min-len", type=int, default=512)
    p.add_argument("--max-len", type=int, default=8192)
    p.add_argument("--out-tokens", type=int, default=128)
    p.add_argument("--token-budget", type=int, default=16384)
    p.add_argument("--max-running", type=int, default=64)
    p.add_argument("--prefill-blocks", type=int, default=8192)
    p.add_argument("--kill-at", type=float, default=0.0, help="seconds after start: the decode instance dies")
    p.add_argument("--restart-s", type=float, default=0.5, help="until its replacement serves")
    p.add_argument("--decode-blocks", type=int, default=16384)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--seed", type=int, default=0)
    return p


def run_serving(args, world: int, rank: int, local: int, cpu) -> Optional[Dict]:
    """One serving run on every rank (the process group is up, ``cpu`` is a
    gloo group); rank 0 returns the summary."""
    dev = torch.device("cuda", local)
    summary = None
    role = "prefill" if rank < world // 2 else "decode"
    args.pair = rank % (world // 2)
    cfg = LlamaConfig(layers=args.layers)
    weights = LlamaWeights.random(cfg, dev, seed=args.seed)
    ctx = zmq.Context()
    sock = ctx.socket(zmq.PAIR)
    port = 29700 + args.pair
    mine = None
    if role == "decode":
        cache = PagedKVCache(cfg, args.decode_blocks, dev)
        ready = torch.zeros(16, dtype=torch.int32, device=dev)
        mine = {"kv": export_tensor(cache.kv).to_dict(), "ready": export_tensor(ready).to_dict(),
                "blocks": args.decode_blocks, "layer_stride": cache.layer_stride_bytes,
                "kv_stride": cache.kv_stride_bytes}
    allx = [None] * world
    dist.all_gather_object(allx, mine, group=cpu)
    mapper = PeerMapper(local)
    if role == "prefill":
        sock.bind(f"tcp://127.0.0.1:{port}")
        d = allx[rank + world // 2]
        dst = KVDestination(base=mapper.open(PeerHandle.from_dict(d["kv"])), layer_stride=d["layer_stride"],
                            kv_stride=d["kv_stride"], heads=cfg.kv_heads, num_blocks=d["blocks"],
                            ready_addr=mapper.open(PeerHandle.from_dict(d["ready"])))
    else:
        sock.connect(f"tcp://127.0.0.1:{port}")
    dist.barrier(group=cpu)
    if role == "prefill":
        res = prefill_side(args, cfg, weights, dev, sock, dst, args.decode_blocks)
    else:
        res = decode_side(args, cfg, weights, dev, sock, cache, ready)
    torch.cuda.synchronize()
    res["role"] = role
    allr = [None] * world
    dist.all_gather_object(allr, res, group=cpu)
    if rank == 0:
        dec = [r for r in allr if r["role"] == "decode"]
        pre = [r for r in allr if r["role"] == "prefill"]
        ttft = [x for r in dec for x in r["ttft_ms"]]
        tpot = [x for r in dec for x in r["tpot_ms"]]
        out_tok = sum(r["output_tokens"] for r in dec)
        span = max(r["span_s"] for r in dec)
        summary = {
            "bench": "pd_serving", "model": f"Llama-3-8B architecture ({args.layers} layers)",
            "pairs": world // 2, "qps_per_pair": args.qps, "duration_s": args.duration,
            "prompt_len": [args.min_len, args.max_len], "out_tokens": args.out_tokens,
            "requests": sum(r["requests"] for r in pre), "completed": sum(r["completed"] for r in dec),
            "ttft_p50_ms": round(_pct(ttft, 50), 2), "ttft_p99_ms": round(_pct(ttft, 99), 2),
            "tpot_p50_ms": round(_pct(tpot, 50), 3), "output_tok_s": round(out_tok / span, 1),
            "kv_push_gbps": round(sum(r["push_bytes"] for r in pre) / max(1e-9, sum(r["push_ms"] for r in pre)) / 1e6, 1),
            "prefill_batches": sum(r["batches"] for r in pre),
            **({"decode_killed_at_s": args.kill_at, "restart_s": args.restart_s,
                "lost_requests": sum(r["lost"] for r in dec), "repushed": sum(r["repushed"] for r in pre),
                "resume_stall_p50_ms": round(_pct([x for r in dec for x in r["stall_ms"]], 50), 1),
                "resume_stall_max_ms": round(max([x for r in dec for x in r["stall_ms"]] or [float("nan")]), 1)}
               if args.kill_at > 0 else {}),
            "decode_steps": sum(r["decode_steps"] for r in dec),
            "data": "synthetic (random token ids, random-init weights)"}
    sock.close(0)
    ctx.term()
    mapper.close()
    dist.barrier(group=cpu)          # every peer mapping is closed before the decode caches go
    return summary if rank == 0 else None



def main() -> None:
    args = parser().parse_args()
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2 or world % 2:
        raise SystemExit("PD serving needs prefill/decode pairs: an even number of GPUs >= 2")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=300))
    out = run_serving(args, world, rank, local, cpu)
    if out is not None:
        print(json.dumps(out), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

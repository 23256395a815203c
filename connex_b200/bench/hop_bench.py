"""Pipeline hop latency between two GPUs: the GPU-driven NVLink channel
(:mod:`connex_b200.parallel.p2pchan`) against NCCL send/recv.

Ping-pong of ``[tokens, 4096]`` bf16 activations (16 KB ... 32 MB) between
rank 0 and rank 1; one-way hop = round trip / 2, device time on rank 0's
stream (CUDA events around ``--iters`` round trips after warm-up; the
receive waits are on the device, so the events span the whole exchange).
Each size is checked for correctness first.  Launch with two processes.
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from connex_b200.parallel.p2pchan import ChanLinks

SIZES = (16 << 10, 1 << 20, 8 << 20, 32 << 20)


def _rtt(send, recv, rank, iters, warmup, dev):
    def once():
        if rank == 0:
            send()
            recv()
        else:
            recv()
            send()
    for _ in range(warmup):
        once()
    torch.cuda.synchronize(dev)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        once()
    b.record()
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) * 1000.0 / iters / 2       # one-way us


def main() -> None:
    import argparse
    p = argparse.ArgumentParser()
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    a = p.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    assert world == 2, "two processes"
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    store = dist.distributed_c10d._get_default_store()
    me, peer = f"hop{rank}", f"hop{1 - rank}"
    chans = ChanLinks(dist.PrefixStore("hop/", store), me, dev)
    res = {}
    for nbytes in SIZES:
        tok = nbytes // (4096 * 2)
        g = torch.Generator(device=dev)
        g.manual_seed(nbytes)                  # the same x on both ranks: rank 1 checks what arrived
        x = torch.randn(tok, 4096, device=dev, generator=g).bfloat16()
        y = torch.empty_like(x)
        if rank == 0:
            tx, rx = chans.open_tx(peer), chans.open_rx(peer)
        else:
            rx, tx = chans.open_rx(peer), chans.open_tx(peer)

        def c_send():
            tx.send([y if rank == 1 else x])
            torch.cuda.current_stream(dev).wait_event(tx.done_event())

        def c_recv():
            rx.recv([y])
            torch.cuda.current_stream(dev).wait_event(rx.done_event())
        # correctness: one transfer 0 -> 1
        c_send() if rank == 0 else c_recv()
        torch.cuda.synchronize(dev)
        ok = bool(torch.equal(y, x)) if rank == 1 else True
        t_chan = _rtt(c_send, c_recv, rank, a.iters, a.warmup, dev)
        chans.check()

        def n_send():
            dist.send(x if rank == 0 else y, 1 - rank)

        def n_recv():
            dist.recv(y, 1 - rank)
        t_nccl = _rtt(n_send, n_recv, rank, a.iters, a.warmup, dev)
        res[nbytes] = {"chan_us": t_chan, "nccl_us": t_nccl, "ok": ok}
    allr = [None, None]
    dist.all_gather_object(allr, res)
    if rank == 0:
        out = {str(k): {"chan_us": round(max(r[k]["chan_us"] for r in allr), 2),
                        "nccl_us": round(max(r[k]["nccl_us"] for r in allr), 2),
                        "correct": all(r[k]["ok"] for r in allr)} for k in SIZES}
        print(json.dumps({"pp_hop_one_way": out, "n_gpus": 2}), flush=True)
    dist.barrier()
    chans.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

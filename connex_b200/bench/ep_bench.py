"""EP MoE layer benchmark: fused peer-memory path vs an NCCL baseline.

Workload (Qwen3-30B-A3B-style MoE layer): hidden 2048, 128 experts, top-8,
expert FFN 768, EP = world size (128 / N experts per rank), bf16, router
logits ~ N(0, 1) plus a Zipf(1.2) popularity bias over experts (seeded),
T tokens per rank.  Measures one full MoE layer (dispatch + expert GEMMs +
combine) per step:

* ``cx``   -- this package's five kernels over NVLink peer memory (no NCCL);
  the per-phase split (count, dispatch, gate/up, down + combine stores,
  combine) comes from CUDA events between the phases on the rank's stream
  (each phase's time includes its wait for the peers);
* ``nccl`` -- the conventional EP layer on NCCL, without host syncs in the
  expert math: per-(rank, expert) counts by ``all_to_all_single``, one host
  read of the split sizes (``all_to_all_single`` with uneven splits needs
  them), tokens sorted by expert and sent with one ``all_to_all_single``,
  the experts as two grouped GEMMs (``torch._grouped_mm`` over per-expert
  offsets on the device), one ``all_to_all_single`` back and a weighted
  ``index_add`` combine.

Device time by CUDA events around ``iters`` steps after warm-up, max over
ranks.  Both paths are checked against each other before timing.
"""
from __future__ import annotations

import statistics
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from connex_b200 import ops
from connex_b200.parallel.ep import EPBuffers, EPConfig, EPMoE, map_remote, peer_table
from connex_b200.parallel.peer import PeerMapper

H, FFN, E, TOPK = 2048, 768, 128, 8


def zipf_routing(T: int, seed: int, device, skew: float = 1.2):
    rng = np.random.default_rng(seed)
    ranks = rng.permutation(E) + 1
    bias = torch.tensor(-skew * np.log(ranks), dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    logits = torch.randn(T, E, generator=g, device=device) + bias
    w, idx = torch.topk(torch.softmax(logits, -1), TOPK, dim=-1)
    return idx.to(torch.int32).contiguous(), (w / w.sum(-1, keepdim=True)).float().contiguous()


def make_weights(S: int, rank: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(1000 + rank)
    gate = torch.randn(S, FFN, H, generator=g, device=device) * 0.02
    up = torch.randn(S, FFN, H, generator=g, device=device) * 0.02
    w13 = torch.stack([ops.interleave_gate_up(gate[i].bfloat16(), up[i].bfloat16()) for i in range(S)]).contiguous()
    w2 = (torch.randn(S, H, FFN, generator=g, device=device) * 0.02).bfloat16().contiguous()
    return w13, w2


_GROUPED_MM: Optional[bool] = None


def _grouped_mm_ok(device) -> bool:
    """Whether ``torch._grouped_mm`` runs here (bf16, jagged M, 3-D weights)."""
    global _GROUPED_MM
    if _GROUPED_MM is None:
        try:
            a = torch.randn(64, 256, device=device).bfloat16()
            b = torch.randn(2, 128, 256, device=device).bfloat16()
            offs = torch.tensor([16, 64], dtype=torch.int32, device=device)
            out = torch._grouped_mm(a, b.transpose(1, 2), offs=offs)
            ref = torch.cat([a[:16].float() @ b[0].float().t(), a[16:].float() @ b[1].float().t()])
            _GROUPED_MM = bool((out.float() - ref).abs().max() < 0.5)
        except (AttributeError, RuntimeError, TypeError):
            _GROUPED_MM = False
    return _GROUPED_MM


def _swiglu(gu: torch.Tensor) -> torch.Tensor:
    """gate/up interleaved per 128 rows of the fused weight -> SiLU(g) * u."""
    v = gu.view(-1, 2 * FFN // 256, 2, 128)
    return F.silu(v[:, :, 0].reshape(-1, FFN)) * v[:, :, 1].reshape(-1, FFN)


def a2a_moe(x, idx, w, w13, w2, N: int, S: int, group=None):
    """Fair baseline: the conventional NCCL EP layer with grouped expert GEMMs
    and one host read (the split sizes) per layer."""
    T, K = idx.shape
    H_ = x.shape[1]
    flat = idx.flatten().long()                        # global expert = dst * S + local expert
    order = torch.argsort(flat, stable=True)           # by destination rank, then local expert
    send_ec = torch.bincount(flat, minlength=N * S).view(N, S)
    recv_ec = torch.empty_like(send_ec)                # [src, local expert]: rows arriving here
    if N > 1:
        dist.all_to_all_single(recv_ec, send_ec, group=group)
    else:
        recv_ec.copy_(send_ec)
    sizes = torch.cat([send_ec.sum(1), recv_ec.sum(1), recv_ec.sum(0)]).cpu()   # the one host sync
    sc, rc, per_e = sizes[:N].tolist(), sizes[N:2 * N].tolist(), sizes[2 * N:]
    R = sum(rc)
    send_x = x[order // K]
    recv_x = torch.empty(R, H_, dtype=x.dtype, device=x.device)
    if N > 1:
        dist.all_to_all_single(recv_x, send_x, rc, sc, group=group)
    else:
        recv_x.copy_(send_x)
    # rows arrive by source, each source's rows by local expert: regroup by expert
    e_of_row = torch.repeat_interleave(torch.arange(S, device=x.device).repeat(N), recv_ec.flatten(), output_size=R)
    perm = torch.argsort(e_of_row, stable=True)
    xe = recv_x[perm]
    if _grouped_mm_ok(x.device):
        offs = torch.cumsum(recv_ec.sum(0), 0).to(torch.int32)
        h = _swiglu(torch._grouped_mm(xe, w13.transpose(1, 2), offs=offs))
        ye = torch._grouped_mm(h, w2.transpose(1, 2), offs=offs)
    else:                                              # per-expert matmuls on host offsets (no further sync)
        ye = torch.empty_like(xe)
        start = 0
        for e, n in enumerate(per_e.tolist()):
            if n:
                ye[start:start + n] = _swiglu(xe[start:start + n] @ w13[e].t()) @ w2[e].t()
            start += n
    out = torch.empty_like(ye)
    out[perm] = ye
    back = torch.empty_like(send_x)
    if N > 1:
        dist.all_to_all_single(back, out, sc, rc, group=group)
    else:
        back.copy_(out)
    y = torch.zeros(T, H_, dtype=torch.float32, device=x.device)
    y.index_add_(0, order // K, back.float() * w.flatten()[order][:, None])
    return y.to(x.dtype)


def nccl_moe(x, idx, w, w13, w2, N: int, S: int, group=None):
    """The naive per-expert loop (host syncs per expert); kept as a reference
    implementation for tests, not as the timed baseline."""
    T, K = idx.shape
    flat = idx.flatten().long()
    dst = flat // S
    order = torch.argsort(dst, stable=True)
    send_counts = torch.bincount(dst, minlength=N)
    recv_counts = torch.empty_like(send_counts)
    if N > 1:
        dist.all_to_all_single(recv_counts, send_counts, group=group)
    else:
        recv_counts.copy_(send_counts)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    send_x = x[order // K]
    send_e = (flat[order] % S).to(torch.int32)
    recv_x = torch.empty(sum(rc), x.shape[1], dtype=x.dtype, device=x.device)
    recv_e = torch.empty(sum(rc), dtype=torch.int32, device=x.device)
    if N > 1:
        dist.all_to_all_single(recv_x, send_x, rc, sc, group=group)
        dist.all_to_all_single(recv_e, send_e, rc, sc, group=group)
    else:
        recv_x.copy_(send_x)
        recv_e.copy_(send_e)
    out = torch.empty_like(recv_x)
    for e in range(S):
        rows = (recv_e == e).nonzero(as_tuple=True)[0]
        if rows.numel() == 0:
            continue
        xe = recv_x[rows]
        gu = xe @ w13[e].t()
        g_, u_ = gu.view(-1, 2 * FFN // 256, 2, 128)[:, :, 0].reshape(-1, FFN), \
            gu.view(-1, 2 * FFN // 256, 2, 128)[:, :, 1].reshape(-1, FFN)
        out[rows] = (F.silu(g_) * u_) @ w2[e].t()
    back = torch.empty_like(send_x)
    if N > 1:
        dist.all_to_all_single(back, out, sc, rc, group=group)
    else:
        back.copy_(out)
    y = torch.zeros(T, x.shape[1], dtype=torch.float32, device=x.device)
    y.index_add_(0, order // K, back.float() * w.flatten()[order][:, None])
    return y.to(x.dtype)


class FusedEP:
    """One rank's fused EP layer with peers mapped through CUDA IPC."""

    def __init__(self, world: int, rank: int, device, max_tokens: int, cpu_group=None):
        self.world, self.rank = world, rank
        S = E // world
        self.cfg = EPConfig(world, S, H, FFN, TOPK, max_tokens=max_tokens)
        self.bufs = EPBuffers(self.cfg, device)
        self.mapper = PeerMapper(device.index)
        if world > 1:
            allx = [None] * world
            dist.all_gather_object(allx, self.bufs.exports(), group=cpu_group)
            addrs = [self.bufs.addresses() if r == rank else map_remote(allx[r], self.mapper)
                     for r in range(world)]
        else:
            addrs = [self.bufs.addresses()]
        self.peers = peer_table(addrs, device)
        self.w13, self.w2 = make_weights(S, rank, device)
        self.layer = EPMoE(self.cfg, rank, self.bufs, self.peers, self.w13, self.w2)
        self.l2p = torch.arange(E, dtype=torch.int32, device=device).view(E, 1).contiguous()
        self.cnt = torch.ones(E, dtype=torch.int32, device=device)

    def forward(self, x, idx, w, out=None, events=None):
        return self.layer.forward(x, idx, w, self.l2p, self.cnt, out, events=events)

    def close(self):
        self.mapper.close()


PHASES = ("count", "dispatch", "gate_up", "down", "combine")


def _phase_times(fused: "FusedEP", x, idx, w, out, iters: int, warmup: int, barrier) -> Dict[str, float]:
    """Mean device time of each phase of the fused layer: events recorded by
    the single native forward call between its own launches (a phase's time
    includes its waits for the peers, none of it host time between phases)."""
    for _ in range(warmup):
        fused.forward(x, idx, w, out)
    barrier()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(PHASES) + 1)] for _ in range(iters)]
    for row in ev:                       # create the events before they are handed over as raw handles
        for e in row:
            e.record()
    torch.cuda.synchronize()
    for it in range(iters):
        fused.forward(x, idx, w, out, events=ev[it])
    torch.cuda.synchronize()
    return {name: 1000.0 * sum(e[k].elapsed_time(e[k + 1]) for e in ev) / iters for k, name in enumerate(PHASES)}


def _time(fn, iters: int, warmup: int, barrier) -> float:
    for _ in range(warmup):
        fn()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / iters  # us


def run_ep_bench(world: int, rank: int, device, cpu_group=None, nccl_group=None,
                 tokens=(128, 4096), iters: int = 20, warmup: int = 5, failover: bool = False) -> Dict:
    barrier = (lambda: dist.barrier(group=cpu_group)) if world > 1 else (lambda: None)
    fused = FusedEP(world, rank, device, max(tokens), cpu_group)
    res: Dict = {}
    for T in tokens:
        idx, w = zipf_routing(T, seed=7 * rank + T, device=device)
        g = torch.Generator(device=device)
        g.manual_seed(rank + T)
        x = (torch.randn(T, H, generator=g, device=device) * 0.5).bfloat16()
        y_cx = fused.forward(x, idx, w)
        y_ref = nccl_moe(x, idx, w, fused.w13, fused.w2, world, E // world, nccl_group)
        torch.cuda.synchronize()
        ops.check_status(fused.bufs.status, "ep")
        err = (y_cx.float() - y_ref.float()).abs().max().item()
        scale = y_ref.float().abs().max().item() + 1e-6
        y_a2a = a2a_moe(x, idx, w, fused.w13, fused.w2, world, E // world, nccl_group)
        err_a2a = (y_a2a.float() - y_ref.float()).abs().max().item()
        out = torch.empty_like(x)
        t_cx = _time(lambda: fused.forward(x, idx, w, out), iters, warmup, barrier)
        phases = _phase_times(fused, x, idx, w, out, iters, warmup, barrier)
        t_nccl = _time(lambda: a2a_moe(x, idx, w, fused.w13, fused.w2, world, E // world, nccl_group),
                       iters, warmup, barrier)
        ops.check_status(fused.bufs.status, "ep")
        res[T] = {"cx_us": t_cx, "nccl_us": t_nccl, "max_err": max(err, err_a2a), "scale": scale,
                  **{f"phase_{k}_us": v for k, v in phases.items()}}
    if failover and world > 1:
        res["failover_ms"] = ep_failover_ms(fused, world, rank, device, barrier, x, idx, w)
    fused.close()
    return res


def ep_failover_ms(fused: "FusedEP", world: int, rank: int, device, barrier, x, idx, w) -> float:
    """The last rank leaves between forwards; the others learn it from the
    store, stop routing to its experts, mark it dead in the EP layer (no
    rebuild) and run the next forward.  Returns leave -> that forward done
    (host clock of the box, ms); the leaving rank returns 0."""
    import time
    store = dist.distributed_c10d._get_default_store()
    victim = world - 1
    barrier()
    torch.cuda.synchronize(device)
    if rank == victim:
        store.set("ep_failover/t", repr(time.time()))
        return 0.0
    store.wait(["ep_failover/t"])
    t_leave = float(store.get("ep_failover/t"))
    S = E // world
    cnt = fused.cnt.clone()
    cnt[victim * S:(victim + 1) * S] = 0          # its experts are no longer routable
    fused.layer.mark_dead(victim)
    fused.layer.forward(x, idx, w, fused.l2p, cnt)
    torch.cuda.synchronize(device)
    ops.check_status(fused.bufs.status, "ep after failover")
    return (time.time() - t_leave) * 1e3


def reduce_max(per_rank: List[Dict]) -> Dict:
    out = {}
    for T in [k for k in per_rank[0] if k != "failover_ms"]:
        keys = ("cx_us", "nccl_us", "max_err", "scale") + tuple(f"phase_{p}_us" for p in PHASES)
        out[str(T)] = {k: max(r[T][k] for r in per_rank) for k in keys if k in per_rank[0][T]}
        out[str(T)]["speedup_vs_nccl"] = round(out[str(T)]["nccl_us"] / out[str(T)]["cx_us"], 2)
        out[str(T)] = {k: (float(f"{v:.4g}") if isinstance(v, float) else v) for k, v in out[str(T)].items()}
    return out


def main() -> None:
    import argparse
    import json
    import os
    from datetime import timedelta
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", default="128,4096")
    p.add_argument("--iters", type=int, default=20)
    a = p.parse_args()
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cpu = nccl = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    res = run_ep_bench(world, rank, dev, cpu, nccl, tokens=tuple(int(t) for t in a.tokens.split(",")),
                       iters=a.iters)
    allr = [None] * world
    if world > 1:
        dist.all_gather_object(allr, res, group=cpu)
    else:
        allr = [res]
    if rank == 0:
        print(json.dumps({"ep_layer_us": reduce_max(allr), "n_gpus": world}), flush=True)
    if world > 1:
        dist.barrier(group=cpu)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""RL weight broadcast inside one NVLink/NVSwitch box, fused with the
trainer -> engine conversion.

The trainer holds unfused HF-named weights (fp32 master or bf16); the
serving engine runs on bf16 weights with q|k|v rows concatenated and gate/up
rows interleaved in blocks of ``GATE_UP_TILE / 2`` (the fused SiLU-mul GEMM
layout).  Conventional sync casts and re-lays out on the trainer, then
broadcasts the bytes.  Here one kernel (``wsync.cu``) does all three: it
reads each trainer tensor once, converts it in registers and stores every
16 bytes through an NVLink multicast address into the live weight arena of
every GPU of the group (NVSwitch replicates the store), then releases a flag
word on every receiver; receivers wait on that flag on their own stream.
Without multicast support it stores to each receiver's arena through its
peer address instead.

The weight arena is symmetric memory (``torch.distributed._symmetric_memory``)
laid out by :func:`engine_manifest`; a receiver's :class:`LlamaWeights` are
views into it (:meth:`LlamaWeights.from_arena`), so an update lands with no
staging copy and no second weight buffer.

Same job of the reference: ``connex/rl/sync.py:41-84`` (publish) and
``:132-259`` (pull + apply) move the bytes; the cast and fused re-layout
there happen in the engine's ``load_weights``.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

from connex.rl.weights import WeightManifest
from connex_b200 import ops
from connex_b200.utils.nvtx import nvtx_range
from connex_b200.models.llama import LlamaConfig, LlamaWeights

WS_COLS = 12
TASK_BYTES = 64 << 10       # output bytes per task (one CTA iteration)
FLAG_BYTES = 4096           # tail of the arena holding the receive flag


def engine_manifest(cfg: LlamaConfig) -> WeightManifest:
    return WeightManifest.build(0, ((n, torch.empty(s, dtype=torch.bfloat16, device="meta"))
                                    for n, s in LlamaWeights.layout(cfg)))


def _targets(cfg: LlamaConfig, name: str):
    """Trainer tensor -> (engine tensor, blk, blk_stride, blk_off) or None (same name, plain copy)."""
    half = ops.GATE_UP_TILE // 2
    hd = cfg.head_dim
    if name.endswith("self_attn.q_proj.weight"):
        return name.replace("q_proj", "qkv_proj"), None, 0, 0
    if name.endswith("self_attn.k_proj.weight"):
        return name.replace("k_proj", "qkv_proj"), None, 0, cfg.heads * hd
    if name.endswith("self_attn.v_proj.weight"):
        return name.replace("v_proj", "qkv_proj"), None, 0, (cfg.heads + cfg.kv_heads) * hd
    if name.endswith("mlp.gate_proj.weight"):
        return name.replace("gate_proj", "gate_up_proj"), half, 2 * half, 0
    if name.endswith("mlp.up_proj.weight"):
        return name.replace("up_proj", "gate_up_proj"), half, 2 * half, half
    return name, None, 0, 0


def plan_jobs(cfg: LlamaConfig, manifest: WeightManifest, src: Dict[str, torch.Tensor],
              task_bytes: int = TASK_BYTES) -> Tuple[torch.Tensor, int, List[torch.Tensor]]:
    """Job table (int64 [n, WS_COLS]) moving every trainer tensor of ``src``
    into the engine arena layout of ``manifest``; returns (jobs, n_tasks, sources)."""
    rows_out: List[List[int]] = []
    srcs: List[torch.Tensor] = []
    task0 = 0
    for name, t in src.items():
        tgt, blk, bstride, boff = _targets(cfg, name)
        e = manifest.entry(tgt)
        if t.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"{name}: {t.dtype} (fp32 or bf16 expected)")
        t2 = t.view(1, -1) if t.dim() == 1 else t
        if t2.dim() != 2 or t2.stride(1) != 1:
            raise ValueError(f"{name}: expected a row-major 2-D (or 1-D) tensor")
        rows, cols = t2.shape
        dcols = e.shape[-1] if len(e.shape) == 2 else e.shape[0]
        if cols != dcols:
            raise ValueError(f"{name}: {cols} columns, engine tensor {tgt} has {dcols}")
        blk = blk or rows
        rpt = max(1, min(rows, task_bytes // (2 * cols)))
        rows_out.append([t2.data_ptr(), e.offset, rows, cols, t2.stride(0), dcols, blk, bstride, boff,
                         int(t.dtype == torch.float32), task0, rpt])
        srcs.append(t2)
        task0 += -(-rows // rpt)
    return torch.tensor(rows_out, dtype=torch.int64), task0, srcs


def emulate_jobs(jobs: torch.Tensor, srcs: Sequence[torch.Tensor], dst_bytes: int) -> torch.Tensor:
    """The kernel's data movement restated in PyTorch (uint8 arena out)."""
    out = torch.zeros(dst_bytes, dtype=torch.uint8)
    for row, s in zip(jobs.tolist(), srcs):
        _, doff, rows, cols, _, dld, blk, bstride, boff, _, _, _ = row
        r = torch.arange(rows)
        drow = (r // blk) * bstride + r % blk + boff
        view = out[doff:].view(torch.bfloat16)
        idx = (drow[:, None] * dld + torch.arange(cols)[None, :]).reshape(-1)
        view[idx] = s.detach().cpu().to(torch.bfloat16).reshape(-1)
    return out


def fuse_reference(cfg: LlamaConfig, named: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Trainer tensors -> engine tensors (bf16, fused layouts) with PyTorch ops."""
    out: Dict[str, torch.Tensor] = {}
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        out[a + "qkv_proj.weight"] = torch.cat([named[a + "q_proj.weight"], named[a + "k_proj.weight"],
                                                named[a + "v_proj.weight"]]).to(torch.bfloat16)
        m = p + "mlp."
        out[m + "gate_up_proj.weight"] = ops.interleave_gate_up(named[m + "gate_proj.weight"].to(torch.bfloat16),
                                                                named[m + "up_proj.weight"].to(torch.bfloat16))
    for n, t in named.items():
        tgt = _targets(cfg, n)[0]
        if tgt == n:
            out[n] = t.to(torch.bfloat16)
    return out


def n_ctas(n_tasks: int, device) -> int:
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return min(n_tasks, 4 * sms)


def apply_local(jobs_cpu: torch.Tensor, dst: torch.Tensor, flag_addr: int = 0) -> int:
    """Fused cast + re-layout of the job sources into the local uint8 arena ``dst``."""
    ops._n()
    jobs_dev = jobs_cpu.to(dst.device)
    return ops._C.wsync(jobs_dev, jobs_cpu, dst.numel(), [dst.data_ptr()], [flag_addr] if flag_addr else [], 0, 0, 0)


class WeightBroadcast:
    """One symmetric weight arena per GPU of ``group``; rank ``src`` sends.

    Collective: every rank constructs it and calls :meth:`sync` together.
    ``mode``: ``"auto"`` (multicast when the GPUs support it, else peer
    stores), ``"multicast"`` or ``"p2p"``.
    """

    def __init__(self, cfg: LlamaConfig, group=None, src: int = 0, device=None, mode: str = "auto",
                 timeout_s: float = 10.0):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.cfg = cfg
        self.group = group or dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.src = src
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.manifest = engine_manifest(cfg)
        self.total = self.manifest.total
        self.timeout_s = timeout_s
        self.arena = symm.empty(self.total + FLAG_BYTES, dtype=torch.uint8, device=self.device)
        self.arena[self.total:].zero_()
        torch.cuda.synchronize(self.device)
        self.handle = symm.rendezvous(self.arena, self.group)
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if mode == "multicast" and not mc:
            raise RuntimeError("NVLink multicast is not available on this group")
        self.mc = mc if mode in ("auto", "multicast") else 0
        self.peers = [int(p) for p in self.handle.buffer_ptrs]
        self.weights = LlamaWeights.from_arena(cfg, self.arena[:self.total], self.manifest)
        self.status = ops.new_status(self.device)
        self.received = 0          # cumulative flag target on this rank
        self._jobs = None
        dist.barrier(group=self.group)

    @property
    def flag_addr(self) -> int:
        return self.arena.data_ptr() + self.total

    def _plan(self, named: Dict[str, torch.Tensor]):
        jobs, n_tasks, srcs = plan_jobs(self.cfg, self.manifest, named)
        return jobs, jobs.to(self.device), n_tasks, srcs

    def sync(self, named: Optional[Dict[str, torch.Tensor]] = None, n_tasks: Optional[int] = None) -> None:
        with nvtx_range("weight broadcast"):
            self._sync(named, n_tasks)

    def _sync(self, named: Optional[Dict[str, torch.Tensor]] = None, n_tasks: Optional[int] = None) -> None:
        """Broadcast ``named`` (src rank) into every rank's arena.

        ``n_tasks`` is the plan's task count (:func:`plan_jobs`); pass it on
        every rank, or None on every rank to have src broadcast it first.
        Stream-ordered: returns once the work is enqueued on every rank."""
        import torch.distributed as dist
        planned = None
        if self.rank == self.src:
            if self._jobs is None or self._jobs[4] is not named:
                jobs, jobs_dev, nt, srcs = self._plan(named)
                self._jobs = (jobs, jobs_dev, nt, srcs, named)
            planned = self._jobs[2]
        if n_tasks is None:
            box = [planned]
            dist.broadcast_object_list(box, src=dist.get_global_rank(self.group, self.src), group=self.group)
            n_tasks = box[0]
        elif planned is not None and planned != n_tasks:
            raise ValueError(f"n_tasks {n_tasks} does not match the plan ({planned})")
        ctas = n_ctas(n_tasks, self.device)
        dist.barrier(group=self.group)      # receivers are off their weights from here on
        if self.rank == self.src:
            jobs, jobs_dev = self._jobs[0], self._jobs[1]
            ops._n()
            if self.mc:
                ops._C.wsync(jobs_dev, jobs, self.total, [], [], self.mc, self.mc + self.total, 0)
            else:
                dst = [p for r, p in enumerate(self.peers) if r != self.rank]
                ops._C.wsync(jobs_dev, jobs, self.total, dst, [p + self.total for p in dst], 0, 0, 0)
            if self.mc:
                self.received += ctas    # the multicast flag store reaches this GPU too
        else:
            self.received += ctas
            ops.wait_flag(self.flag_addr, self.received & 0xFFFFFFFF, self.status, self.timeout_s)

    def check(self) -> None:
        ops.check_status(self.status, "weight broadcast")

    def close(self) -> None:
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

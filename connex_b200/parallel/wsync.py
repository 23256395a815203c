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
FLAG_BYTES = 4096           # tail of the arena holding the receive flags
RELAY_FLAG = 64             # byte offset (in that tail) of the relay-round flag
RELAY_ROUNDS = 16           # rounds a relayed broadcast is cut into


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


def shard_dim0(named: Dict[str, torch.Tensor], rank: int, world: int,
               align: int = ops.GATE_UP_TILE // 2) -> Tuple[Dict[str, torch.Tensor], Dict[str, int]]:
    """Per-parameter dim-0 shards of ``named`` (FSDP2 ``Shard(0)``) held by
    trainer ``rank`` of ``world``: ``(local views, global start of each)``.
    Row boundaries are multiples of ``align`` rows (1-D tensors: of 8
    elements), so every shard starts on a gate/up block and a 16-byte column."""
    local, start = {}, {}
    for name, t in named.items():
        n = t.shape[0]
        unit = 8 if t.dim() == 1 else align
        per = -(-n // (world * unit)) * unit
        a, b = min(n, rank * per), min(n, (rank + 1) * per)
        if a < b:
            local[name], start[name] = t[a:b], a
    return local, start


def plan_jobs(cfg: LlamaConfig, manifest: WeightManifest, src: Dict[str, torch.Tensor],
              task_bytes: int = TASK_BYTES, starts: Optional[Dict[str, int]] = None
              ) -> Tuple[torch.Tensor, int, List[torch.Tensor]]:
    """Job table (int64 [n, WS_COLS]) moving every trainer tensor of ``src``
    into the engine arena layout of ``manifest``; returns (jobs, n_tasks, sources).

    ``starts`` (sharded trainers): the global first row (1-D: first element)
    of each local tensor.  The shard's place in the engine tensor is folded
    into the job's destination offset, so the kernel is the same for a whole
    tensor and for a shard."""
    rows_out: List[List[int]] = []
    srcs: List[torch.Tensor] = []
    task0 = 0
    starts = starts or {}
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
        s0 = int(starts.get(name, 0))
        doff = e.offset
        if t.dim() == 1:
            if s0 % 8 or s0 + cols > dcols:
                raise ValueError(f"{name}: shard [{s0}, +{cols}) does not fit {tgt} ({dcols}) on 8-element bounds")
            doff += 2 * s0
        else:
            if cols != dcols:
                raise ValueError(f"{name}: {cols} columns, engine tensor {tgt} has {dcols}")
            if blk is not None:
                if s0 % blk:
                    raise ValueError(f"{name}: shard start {s0} is not on a {blk}-row block")
                doff += 2 * (s0 // blk) * bstride * dcols
            else:
                doff += 2 * s0 * dcols
        blk = blk or rows
        rpt = max(1, min(rows, task_bytes // (2 * cols)))
        rows_out.append([t2.data_ptr(), doff, rows, cols, t2.stride(0), dcols, blk, bstride, boff,
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


# ------------------------------------------------------------- relay plans
def job_intervals(jobs_cpu: torch.Tensor) -> List[Tuple[int, int]]:
    """Destination byte intervals ``(offset, nbytes)`` the job rows write,
    sorted and merged (a job whose rows are interleaved in blocks writes one
    interval per block)."""
    out = []
    for _, doff, rows, cols, _, dld, blk, bstride, boff, _, _, _ in jobs_cpu.tolist():
        if cols != dld:
            raise ValueError("relay plans need jobs that write whole destination rows")
        row_b = 2 * dld
        if blk >= rows:
            out.append((doff + boff * row_b, rows * row_b))
        else:
            for i in range(0, rows, blk):
                out.append((doff + ((i // blk) * bstride + boff) * row_b, min(blk, rows - i) * row_b))
    out.sort()
    merged: List[Tuple[int, int]] = []
    for off, n in out:
        if merged and merged[-1][0] + merged[-1][1] == off:
            merged[-1] = (merged[-1][0], merged[-1][1] + n)
        else:
            merged.append((off, n))
    return merged


def split_intervals(intervals: Sequence[Tuple[int, int]], slice_bytes: int, n: int) -> List[List[Tuple[int, int]]]:
    """The intervals cut at slice boundaries: per slice owner (the last owner
    takes everything past ``(n - 1) * slice_bytes``)."""
    per: List[List[Tuple[int, int]]] = [[] for _ in range(n)]
    for off, ln in intervals:
        end = off + ln
        while off < end:
            k = min(off // slice_bytes, n - 1)
            stop = end if k == n - 1 else min(end, (k + 1) * slice_bytes)
            per[k].append((off, stop - off))
            off = stop
    return per


def copy_jobs(intervals: Sequence[Tuple[int, int]], base: int, task_bytes: int = TASK_BYTES
              ) -> Tuple[torch.Tensor, int]:
    """Identity bf16 copy jobs reading ``base + offset`` for each interval and
    writing the same offsets (the relay's forward of its slice)."""
    rows_out, task0 = [], 0
    for off, n in intervals:
        el = n // 2
        cols = next(c for c in (4096, 2048, 1024, 512, 256, 128, 64, 32, 16, 8) if el % c == 0)
        rows = el // cols
        rpt = max(1, min(rows, task_bytes // (2 * cols)))
        rows_out.append([base + off, off, rows, cols, cols, cols, rows, 0, 0, 0, task0, rpt])
        task0 += -(-rows // rpt)
    if not rows_out:
        return torch.zeros(0, WS_COLS, dtype=torch.int64), 0
    return torch.tensor(rows_out, dtype=torch.int64), task0


def split_rounds(jobs_cpu: torch.Tensor, rounds: int) -> List[torch.Tensor]:
    """Whole job rows grouped into ``rounds`` consecutive groups of about equal
    output bytes, each with its own running task prefix."""
    rows = jobs_cpu.tolist()
    total = sum(r[2] * r[3] * 2 for r in rows)
    groups, cur, acc = [], [], 0
    for r in rows:
        cur.append(list(r))
        acc += r[2] * r[3] * 2
        if acc >= total * (len(groups) + 1) / rounds and len(groups) < rounds - 1:
            groups.append(cur)
            cur = []
    if cur:
        groups.append(cur)
    out = []
    for g in groups:
        t = 0
        for r in g:
            r[10] = t
            t += -(-r[2] // r[11])
        out.append(torch.tensor(g, dtype=torch.int64))
    return out


def _tasks(jobs_cpu: torch.Tensor) -> int:
    return sum(-(-r[2] // r[11]) for r in jobs_cpu.tolist())


def n_ctas(n_tasks: int, device) -> int:
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return min(n_tasks, 4 * sms)


def apply_local(jobs_cpu: torch.Tensor, dst: torch.Tensor, flag_addr: int = 0) -> int:
    """Fused cast + re-layout of the job sources into the local uint8 arena ``dst``."""
    ops._n()
    jobs_dev = jobs_cpu.to(dst.device)
    return ops._C.wsync(jobs_dev, jobs_cpu, dst.numel(), [dst.data_ptr()], [flag_addr] if flag_addr else [], 0, 0, 0)


class WeightBroadcast:
    """One symmetric weight arena per GPU of ``group``; the ranks in ``srcs``
    (trainer shards, or one trainer) send.

    Collective: every rank constructs it and calls :meth:`sync` together.
    ``mode``: ``"auto"`` (multicast when the GPUs support it and there is
    more than one receiver, else peer stores), ``"multicast"`` or ``"p2p"``.

    ``"relay"`` (one trainer, every other rank a member): the trainer stores
    each 16-byte piece only into the receiver that owns its slice of the
    arena (its egress is the model size once, at the unicast link rate), in
    ``RELAY_ROUNDS`` rounds; as soon as a round has landed, each receiver
    multicasts its share of that round to every arena.  Measured on 8 B200:
    one trainer multicasting to 7 receivers is limited by the switch's
    replication (16 GB in 39 ms), the scatter alone takes 23 ms and the
    receivers' concurrent multicasts of their slices 25 ms; run together
    (per-round events, ``wsync_bench --relay-timeline``) the forwards lag the
    scatter by up to 10 ms a round and the whole takes 45 ms, since every
    receiver's ingress carries its own multicast echo and six others' shares
    while the scatter competes for it.  ``"relay_p2p"`` forwards with peer
    stores to the other receivers instead (no echo, no switch replication);
    measured on 8 B200 it is slower still (53.9 ms against 46.1 ms relay,
    40.0 ms one-source multicast and 40.4 ms NCCL), with the same lagging
    forwards: the receivers' ingress under the concurrent scatter, not the
    multicast, sets the time.  ``"auto"`` stays one-source multicast.

    Membership per round (``sync(members=...)``): in multicast mode NVSwitch
    delivers every round to every GPU bound to the group, so a rank that
    stopped consuming (left) blocks nobody, and a standby rank that joins
    already holds the latest version once its flag shows the round; in p2p
    mode only the round's members are written, and a rank that joins later
    catches up with :meth:`catch_up` (one ``copy_segments`` launch reading a
    member's arena over NVLink).  No sender ever waits for a receiver.
    """

    def __init__(self, cfg: LlamaConfig, group=None, src: int = 0, device=None, mode: str = "auto",
                 timeout_s: float = 10.0, srcs: Optional[Sequence[int]] = None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.cfg = cfg
        self.group = group or dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.srcs = list(srcs) if srcs is not None else [src]
        self.src = self.srcs[0]
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.manifest = engine_manifest(cfg)
        self.total = self.manifest.total
        self.timeout_s = timeout_s
        self.arena = symm.empty(self.total + FLAG_BYTES, dtype=torch.uint8, device=self.device)
        self.arena.zero_()          # padding between tensors included: arenas compare bytewise
        torch.cuda.synchronize(self.device)
        self.handle = symm.rendezvous(self.arena, self.group)
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if mode in ("multicast", "relay") and not mc:
            raise RuntimeError("NVLink multicast is not available on this group")
        if mode in ("relay", "relay_p2p") and len(self.srcs) != 1:
            raise ValueError("relay mode has one source")
        self.relay = mode in ("relay", "relay_p2p")
        # relay_p2p: receivers pass their share on with peer stores to the
        # other receivers instead of one multicast store to every arena
        self.relay_p2p = mode == "relay_p2p"
        # auto: multicast, except with a single receiver, where plain peer
        # stores measured faster (8 B200, 16 GB: 23.1 ms against 28.9 ms; from
        # three receivers up multicast wins, 29.2 against 67.3 ms)
        single_receiver = self.world - len(self.srcs) == 1
        self.mc = mc if mode in ("multicast", "relay") or (mode == "auto" and not single_receiver) else 0
        self.peers = [int(p) for p in self.handle.buffer_ptrs]
        self.weights = LlamaWeights.from_arena(cfg, self.arena[:self.total], self.manifest)
        self.status = ops.new_status(self.device)
        self.received = 0          # cumulative flag target on this rank
        self.relay_received = 0    # cumulative target of the relay-round flag
        self._relay = None         # (plan version, per-rank relay state)
        self._plan_version = 0
        self.rounds_seen = 0       # rounds whose flag increments reached this rank
        self.round = 0
        self._jobs = None
        self.timeline: Optional[list] = None   # set to [] to record the relay's per-round events
        dist.barrier(group=self.group)

    @property
    def flag_addr(self) -> int:
        return self.arena.data_ptr() + self.total

    @property
    def relay_flag_addr(self) -> int:
        return self.arena.data_ptr() + self.total + RELAY_FLAG

    @property
    def is_src(self) -> bool:
        return self.rank in self.srcs

    def _plan(self, named: Dict[str, torch.Tensor], starts=None):
        jobs, n_tasks, srcs = plan_jobs(self.cfg, self.manifest, named, starts=starts)
        return jobs, jobs.to(self.device), n_tasks, srcs

    def sync(self, named: Optional[Dict[str, torch.Tensor]] = None, n_tasks=None, starts=None,
             members: Optional[Sequence[int]] = None, wait: bool = True) -> None:
        with nvtx_range("weight broadcast"):
            self._sync(named, n_tasks, starts, members, wait)

    def _sync(self, named, n_tasks, starts, members, wait) -> None:
        """Broadcast every source's ``named`` (its shard, placed by
        ``starts``) into the arenas.

        ``n_tasks``: per source (list, or an int with one source) the plan's
        task count; None on every rank to gather it first.  ``members``: the
        ranks consuming this round (default: every non-source rank);
        ``wait=False``: this rank does not wait for the round (it is
        leaving).  Stream-ordered: returns once the work is enqueued."""
        import torch.distributed as dist
        planned = None
        if self.is_src:
            if self._jobs is None or self._jobs[4] is not named:
                jobs, jobs_dev, nt, srcs = self._plan(named, starts)
                self._jobs = (jobs, jobs_dev, nt, srcs, named)
                self._plan_version += 1
            planned = self._jobs[2]
        recv_all = [r for r in range(self.world) if r not in self.srcs]
        if self.relay and (members is None or sorted(members) == recv_all) and recv_all:
            self._sync_relay(planned, wait)
            return
        if n_tasks is None:
            box = [None] * self.world
            dist.all_gather_object(box, planned, group=self.group)
            n_tasks = [box[r] for r in self.srcs]
        elif isinstance(n_tasks, int):
            n_tasks = [n_tasks]
        if len(n_tasks) != len(self.srcs):
            raise ValueError(f"{len(n_tasks)} task counts for {len(self.srcs)} sources")
        if planned is not None and planned != n_tasks[self.srcs.index(self.rank)]:
            raise ValueError(f"n_tasks {n_tasks} does not match the plan ({planned})")
        ctas = sum(n_ctas(n, self.device) for n in n_tasks)
        members = [r for r in range(self.world) if r not in self.srcs] if members is None else list(members)
        self.round += 1
        dist.barrier(group=self.group)      # receivers are off their weights from here on
        if self.is_src:
            jobs, jobs_dev = self._jobs[0], self._jobs[1]
            ops._n()
            if self.mc:
                ops._C.wsync(jobs_dev, jobs, self.total, [], [], self.mc, self.mc + self.total, 0)
            else:
                dst = [self.peers[r] for r in members if r != self.rank]
                if dst:                        # a round may have no consuming member
                    ops._C.wsync(jobs_dev, jobs, self.total, dst, [p + self.total for p in dst], 0, 0, 0)
        gets_round = bool(self.mc) or self.rank in members
        if gets_round:
            self.received += ctas
            self.rounds_seen = self.round
        if gets_round and wait and not self.is_src and self.rank in members:
            ops.wait_flag(self.flag_addr, self.received & 0xFFFFFFFF, self.status, self.timeout_s)

    def _relay_state(self, planned) -> dict:
        """This rank's part of the relay plan: the trainer's round tables, each
        receiver's forward tables, and the flag arrivals to wait for.  Planned
        on the trainer, shipped once per plan version."""
        import torch.distributed as dist
        box = [None] * self.world
        dist.all_gather_object(box, (planned, self._plan_version) if self.is_src else None, group=self.group)
        planned, version = box[self.src]
        if self._relay is not None and self._relay[0] == version:
            return self._relay[1]
        recv = [r for r in range(self.world) if r != self.src]
        slice_bytes = -(-self.total // (len(recv) * 16)) * 16
        meta = [None]
        if self.is_src:
            rounds = split_rounds(self._jobs[0], RELAY_ROUNDS)
            per_round = [split_intervals(job_intervals(j), slice_bytes, len(recv)) for j in rounds]
            meta = [([_tasks(j) for j in rounds], per_round)]
        dist.broadcast_object_list(meta, src=self.src, group=self.group)
        src_tasks, per_round = meta[0]
        st = {"slice": slice_bytes, "recv": recv, "src_ctas": [n_ctas(t, self.device) for t in src_tasks]}
        fwd_ctas, fwd_by = 0, [0] * len(recv)
        for ivs in per_round:
            for k in range(len(recv)):
                n = n_ctas(copy_jobs(ivs[k], 0)[1], self.device) if ivs[k] else 0
                fwd_ctas += n
                fwd_by[k] += n
        st["fwd_ctas_total"] = fwd_ctas
        st["fwd_by_recv"] = fwd_by
        if self.is_src:
            st["rounds"] = [(j, j.to(self.device)) for j in split_rounds(self._jobs[0], RELAY_ROUNDS)]
        else:
            j = recv.index(self.rank)
            fw = []
            for ivs in per_round:
                jobs, nt = copy_jobs(ivs[j], self.arena.data_ptr())
                fw.append((jobs, jobs.to(self.device) if nt else None))
            st["fwd"] = fw
        self._relay = (version, st)
        return st

    def _sync_relay(self, planned, wait: bool) -> None:
        import torch.distributed as dist
        st = self._relay_state(planned)
        self.round += 1
        dist.barrier(group=self.group)      # receivers are off their weights from here on
        ops._n()
        tl = self.timeline is not None
        if tl:                              # per-round events, relative to this rank's start
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record()
            marks = []

        def mark(tag):
            if tl:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                marks.append((tag, e))
        if self.is_src:
            dst = [self.peers[r] for r in st["recv"]]
            for r, (jobs, jobs_dev) in enumerate(st["rounds"]):
                ops._C.wsync(jobs_dev, jobs, self.total, dst, [p + self.total for p in dst], 0, 0, 0, st["slice"])
                mark(f"scatter{r}")
            if not self.relay_p2p:
                self.relay_received += st["fwd_ctas_total"]  # the multicast forwards land in this arena too
            if tl:
                self._record_timeline(ev0, marks)
            return
        for r, ((jobs, jobs_dev), ctas) in enumerate(zip(st["fwd"], st["src_ctas"])):
            self.received += ctas                            # this round's scatter has landed here...
            ops.wait_flag(self.flag_addr, self.received & 0xFFFFFFFF, self.status, self.timeout_s)
            mark(f"landed{r}")
            if jobs_dev is not None:                         # ...so pass this rank's share on to every arena
                if self.relay_p2p:
                    others = [self.peers[q] for q in st["recv"] if q != self.rank]
                    if others:
                        ops._C.wsync(jobs_dev, jobs, self.total, others,
                                     [b + self.total + RELAY_FLAG for b in others], 0, 0, 0)
                else:
                    ops._C.wsync(jobs_dev, jobs, self.total, [], [], self.mc, self.mc + self.total + RELAY_FLAG, 0)
            mark(f"forwarded{r}")
        if tl:
            self._record_timeline(ev0, marks)
        mine = st["fwd_by_recv"][st["recv"].index(self.rank)]
        # every forward CTA releases each destination once: multicast reaches
        # every arena (this one included), peer stores only the other receivers
        self.relay_received += st["fwd_ctas_total"] - (mine if self.relay_p2p else 0)
        self.rounds_seen = self.round
        if wait:
            ops.wait_flag(self.relay_flag_addr, self.relay_received & 0xFFFFFFFF, self.status, self.timeout_s)

    def _record_timeline(self, ev0, marks) -> None:
        """Milliseconds from this rank's start of the relay to each mark."""
        torch.cuda.synchronize(self.device)
        self.timeline.append({tag: round(ev0.elapsed_time(e), 3) for tag, e in marks})

    def catch_up(self, from_rank: int, max_ctas: int = 64) -> None:
        """Copy member ``from_rank``'s arena (the latest version) into this
        rank's, reading it over NVLink (p2p-mode joiners).  Stream-ordered;
        the caller orders it after that member's round."""
        seg = torch.tensor([[self.peers[from_rank], self.arena.data_ptr(), self.total]], dtype=torch.int64,
                           device=self.device)
        ops.copy_segments(seg, self.total, max_ctas=max_ctas, status=self.status)
        self.rounds_seen = self.round

    def check(self) -> None:
        ops.check_status(self.status, "weight broadcast")

    def close(self) -> None:
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

"""Expert-parallel MoE layer over NVLink peer memory (no NCCL on this path).

Each rank owns ``S`` expert slots (physical slot ``p`` lives on rank
``p // S``); routing goes through the placement table's logical -> physical
map (``l2p [E, R]`` + ``l2p_cnt [E]``, the view an :class:`EPController`
pushes), so migrated or replicated experts are picked up at the next step
without any kernel change.  One forward is five kernels on the rank's
stream (``moe.cu``): count (all-gather of the count matrix), dispatch
(peer stores of token rows + metadata), gate/up grouped GEMM (tcgen05,
SiLU-mul epilogue), down grouped GEMM whose epilogue stores the weighted
rows into the source ranks' combine buffers, and combine.  Cross-rank
ordering uses cumulative u32 counters (one epoch per forward, identical on
every rank), every wait is bounded and reports through ``status``.

:func:`emulated_group` runs N ranks in one process on one GPU (every rank's
buffers are local memory) by issuing each kernel phase for all ranks before
the next phase: each wait is then satisfied by launches that already ran,
so no kernel ever depends on another one running concurrently.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from connex_b200 import _C, ops
from connex_b200.utils.nvtx import nvtx_range

FLAG_COUNT, FLAG_DATA, FLAG_COMB, FLAG_EXPECT = 0, 4, 8, 12  # int32 offsets (16 B apart)


@dataclass
class EPConfig:
    n_ranks: int
    slots_per_rank: int
    hidden: int = 2048
    ffn: int = 768
    top_k: int = 8
    max_tokens: int = 4096  # per rank per forward

    @property
    def recv_rows(self) -> int:
        return self.n_ranks * self.max_tokens * self.top_k


class EPBuffers:
    """Device memory one rank exposes to its peers."""

    def __init__(self, cfg: EPConfig, device):
        N, S, H, K = cfg.n_ranks, cfg.slots_per_rank, cfg.hidden, cfg.top_k
        R = cfg.recv_rows
        self.device = device
        self.counts = torch.zeros(N, N, S, dtype=torch.int32, device=device)
        self.flags = torch.zeros(16, dtype=torch.int32, device=device)
        self.recv = torch.empty(R, H, dtype=torch.bfloat16, device=device)
        self.recv_meta = torch.zeros(R, 4, dtype=torch.int32, device=device)
        self.mid = torch.empty(R, cfg.ffn, dtype=torch.bfloat16, device=device)
        self.comb = torch.empty(cfg.max_tokens * K, H, dtype=torch.bfloat16, device=device)
        self.pos = torch.empty(cfg.max_tokens * K, dtype=torch.int32, device=device)
        self.slot_of = torch.empty(cfg.max_tokens * K, dtype=torch.int32, device=device)
        self.status = ops.new_status(device)

    def flag_addr(self, which: int) -> int:
        return self.flags.data_ptr() + 4 * which

    def addresses(self) -> List[int]:
        """(counts, count_flag, recv, recv_meta, data_flag, comb, comb_flag)."""
        return [self.counts.data_ptr(), self.flag_addr(FLAG_COUNT), self.recv.data_ptr(), self.recv_meta.data_ptr(),
                self.flag_addr(FLAG_DATA), self.comb.data_ptr(), self.flag_addr(FLAG_COMB)]

    def exports(self) -> List[dict]:
        from connex_b200.parallel.peer import export_tensor
        return [export_tensor(t).to_dict() for t in (self.counts, self.flags, self.recv, self.recv_meta, self.comb)]


def peer_table(per_rank: List[List[int]], device) -> torch.Tensor:
    """[7, N] int64 device tensor from each rank's 7 addresses (as seen locally)."""
    return torch.tensor(per_rank, dtype=torch.int64).t().contiguous().to(device)


def map_remote(exports: List[dict], mapper) -> List[int]:
    """Addresses of a remote rank's EP buffers in this process (IPC mappings)."""
    from connex_b200.parallel.peer import PeerHandle
    counts, flags, recv, meta, comb = (mapper.open(PeerHandle.from_dict(e)) for e in exports)
    return [counts, flags + 4 * FLAG_COUNT, recv, meta, flags + 4 * FLAG_DATA, comb, flags + 4 * FLAG_COMB]


class EPMoE:
    """One rank's EP MoE layer: ``forward(x, topk_idx, topk_w, l2p, l2p_cnt)``."""

    def __init__(self, cfg: EPConfig, rank: int, bufs: EPBuffers, peers: torch.Tensor, w13: torch.Tensor,
                 w2: torch.Tensor):
        """``w13`` [S, 2F, H] (gate/up interleaved per 256 rows), ``w2`` [S, H, F]."""
        self.cfg, self.rank, self.b, self.peers = cfg, rank, bufs, peers
        self.w13 = w13.reshape(cfg.slots_per_rank * 2 * cfg.ffn, cfg.hidden)
        self.w2 = w2.reshape(cfg.slots_per_rank * cfg.hidden, cfg.ffn)
        self.epoch = 0
        self.live = [True] * cfg.n_ranks
        self.count_expected = 0      # cumulative u32 targets: + live ranks per forward
        self.data_expected = 0
        self._sink = None
        self._fwd = None             # (combine-expect view, data flag address, combine flag address)

    @property
    def n_live(self) -> int:
        return sum(self.live)

    def mark_dead(self, rank: int) -> None:
        """Stop exchanging with ``rank`` (it left between forwards; every rank
        calls this at the same forward boundary, after its l2p stops routing to
        ``rank``'s slots).  Its column of the peer table points at local sinks
        from now on, so no kernel touches its memory again, its stale row of the
        count matrix is cleared, and the wait targets count live ranks only --
        no buffer is reallocated and no IPC mapping reopened."""
        if not self.live[rank] or rank == self.rank:
            return
        c, b = self.cfg, self.b
        if self._sink is None:
            self._sink = (torch.zeros_like(b.counts), torch.zeros(16, dtype=torch.int32, device=b.device))
        sc, sf = self._sink
        col = torch.tensor([sc.data_ptr(), sf.data_ptr() + 4 * FLAG_COUNT, b.recv.data_ptr(), b.recv_meta.data_ptr(),
                            sf.data_ptr() + 4 * FLAG_DATA, b.comb.data_ptr(), sf.data_ptr() + 4 * FLAG_COMB],
                           dtype=torch.int64, device=self.peers.device)
        self.peers[:, rank] = col
        b.counts[rank].zero_()
        self.live[rank] = False

    # the five phases (separately callable for the single-GPU emulation)
    def phase_count(self, topk_idx, l2p, l2p_cnt):
        c = self.cfg
        if topk_idx.shape[0] > c.max_tokens or topk_idx.shape[1] != c.top_k:
            raise ValueError(f"EP layer holds {c.max_tokens} tokens x top-{c.top_k}; got {tuple(topk_idx.shape)}")
        self.epoch += 1
        self.count_expected = (self.count_expected + self.n_live) & 0xFFFFFFFF
        self.data_expected = (self.data_expected + self.n_live * _C.EP_DISPATCH_CTAS) & 0xFFFFFFFF
        _C.ep_count(topk_idx, l2p, l2p_cnt, c.slots_per_rank, self.rank, self.b.pos, self.b.slot_of, self.peers,
                    self.b.flags[FLAG_EXPECT:FLAG_EXPECT + 1], c.hidden // 256, self.b.status)
        ops._n()

    def phase_dispatch(self, x, topk_w):
        c = self.cfg
        _C.ep_dispatch(x, topk_w, self.b.pos, self.b.slot_of, self.b.counts, c.top_k, c.slots_per_rank, self.rank,
                       c.recv_rows, self.count_expected, self.peers, self.b.status)
        ops._n()

    def _data_target(self) -> int:
        return self.data_expected

    def phase_gate_up(self):
        c = self.cfg
        _C.ep_grouped_gemm(self.b.recv, self.w13, 2 * c.ffn, self.b.mid, self.b.counts, c.slots_per_rank, self.rank,
                           0, self.b.recv_meta, self.peers, c.hidden, self.b.flag_addr(FLAG_DATA),
                           self._data_target(), self.b.status)
        ops._n()

    def phase_down(self):
        c = self.cfg
        _C.ep_grouped_gemm(self.b.mid, self.w2, c.hidden, self.b.mid, self.b.counts, c.slots_per_rank, self.rank, 1,
                           self.b.recv_meta, self.peers, c.hidden, self.b.flag_addr(FLAG_DATA), self._data_target(),
                           self.b.status)
        ops._n()

    def phase_combine(self, T: int, out: torch.Tensor):
        c = self.cfg
        _C.ep_combine(self.b.comb, self.b.slot_of, T, c.top_k, out, self.b.flag_addr(FLAG_COMB),
                      self.b.flags[FLAG_EXPECT:FLAG_EXPECT + 1], self.b.status)
        ops._n()
        return out

    def forward(self, x, topk_idx, topk_w, l2p, l2p_cnt, out: Optional[torch.Tensor] = None,
                events: Optional[list] = None):
        """The five phases in one native call (``ep_forward``): at a few
        hundred tokens the layer's device work is tens of microseconds, so
        five separate crossings from Python would set its time.  ``events``:
        six recorded-once ``torch.cuda.Event`` (timing) to mark the phase
        boundaries on the stream."""
        c, b = self.cfg, self.b
        if topk_idx.shape[0] > c.max_tokens or topk_idx.shape[1] != c.top_k:
            raise ValueError(f"EP layer holds {c.max_tokens} tokens x top-{c.top_k}; got {tuple(topk_idx.shape)}")
        out = torch.empty_like(x) if out is None else out
        self.epoch += 1
        self.count_expected = (self.count_expected + self.n_live) & 0xFFFFFFFF
        self.data_expected = (self.data_expected + self.n_live * _C.EP_DISPATCH_CTAS) & 0xFFFFFFFF
        if self._fwd is None:
            self._fwd = (b.flags[FLAG_EXPECT:FLAG_EXPECT + 1], b.flag_addr(FLAG_DATA), b.flag_addr(FLAG_COMB))
        expect, data_flag, comb_flag = self._fwd
        with nvtx_range("ep forward"):
            _C.ep_forward(x, topk_idx, topk_w, l2p, l2p_cnt, out, self.w13, self.w2, b.pos, b.slot_of, b.counts,
                          b.recv, b.recv_meta, b.mid, b.comb, expect, self.peers, c.slots_per_rank, self.rank,
                          c.ffn, c.recv_rows, self.count_expected, data_flag, self.data_expected, comb_flag,
                          b.status, [e.cuda_event for e in events] if events else [])
        ops._n(5)
        return out


def emulated_group(cfg: EPConfig, w13_all: torch.Tensor, w2_all: torch.Tensor, device) -> List[EPMoE]:
    """N ranks in one process on one GPU; ``w13_all`` [N*S, 2F, H], ``w2_all`` [N*S, H, F]."""
    N, S = cfg.n_ranks, cfg.slots_per_rank
    bufs = [EPBuffers(cfg, device) for _ in range(N)]
    peers = peer_table([b.addresses() for b in bufs], device)
    return [EPMoE(cfg, r, bufs[r], peers, w13_all[r * S:(r + 1) * S], w2_all[r * S:(r + 1) * S]) for r in range(N)]


def emulated_forward(layers: List[EPMoE], xs, idxs, ws, l2p, l2p_cnt) -> List[torch.Tensor]:
    """Phase by phase over all emulated ranks (see the module docstring)."""
    for L, i in zip(layers, idxs):
        L.phase_count(i, l2p, l2p_cnt)
    for L, x, w in zip(layers, xs, ws):
        L.phase_dispatch(x, w)
    for L in layers:
        L.phase_gate_up()
    for L in layers:
        L.phase_down()
    return [L.phase_combine(x.shape[0], torch.empty_like(x)) for L, x in zip(layers, xs)]


def reference_moe(x, topk_idx, topk_w, w13_all, w2_all, l2p=None, l2p_cnt=None):
    """fp32 PyTorch MoE: y[t] = sum_k w * down_e(SiLU(gate_e x) * up_e x)."""
    import torch.nn.functional as F
    from connex_b200.ops import deinterleave_gate_up
    T, K = topk_idx.shape
    y = torch.zeros(T, x.shape[1], dtype=torch.float32, device=x.device)
    for t in range(T):
        for k in range(K):
            e = int(topk_idx[t, k])
            if l2p is not None:
                c = int(l2p_cnt[e])
                if c == 0:
                    continue
                e = int(l2p[e, t % c])
            g, u = deinterleave_gate_up(w13_all[e])
            h = F.silu(x[t].float() @ g.float().t()) * (x[t].float() @ u.float().t())
            y[t] += float(topk_w[t, k]) * (h.to(torch.bfloat16).float() @ w2_all[e].float().t())
    return y

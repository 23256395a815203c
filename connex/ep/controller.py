"""EP control plane: owns the placement table and drives the engines through
epochs.

Every reconfiguration -- a rank fails, drains or joins, experts migrate --
is a :class:`_Reconfiguration` of two published epochs:

1. **cutover** (epoch k+1): the table routes around down / draining ranks
   and around the destination slots of the planned moves; every engine
   applies that view;
2. **copy**: the destination ranks pull the expert weights from a live
   replica (from the checkpoint loader when none is left).  A move that
   fails is re-planned from another source for up to ``max_rounds``
   rounds; a source reported unreachable marks its rank down;
3. **commit** (epoch k+2): the destination slots become routable with their
   new experts (failed moves leave them empty); every engine applies.

Engines apply a view only between steps, so no step mixes two placements.
An *engine* handle provides ``apply(view) -> bool`` (False: the view is
older than one it has), ``describe() -> {rank: desc}`` and ``move(moves,
peers, slots_per_rank) -> [(move, ok, err)]``.  :class:`LocalEngine` is the
in-process EP group for tests and demos.  Each reconfiguration returns a
report dict with the phase times (``cutover_s``, ``copy_s``, ``commit_s``,
``total_s``), ``moves``, ``failed_moves``, ``rounds``, ``bytes``, the epochs
and the number of uncovered (layer, expert) pairs left.

Behavioural parity: ``connex/ep/controller.py:36-240`` of the reference.
"""
from __future__ import annotations

import logging
import threading
import time
from typing import Dict, List, Optional

import torch

from connex.ep.placement import Move, PlacementError, PlacementTable, logical_to_physical

log = logging.getLogger("connex.ep")


class _Reconfiguration:
    """One run of the two-epoch protocol over a list of moves."""

    def __init__(self, ctl: "EPController", event: str, moves: List[Move]):
        self.ctl, self.t = ctl, ctl.table
        self.pending = list(moves)
        self.report = {"event": event, "epoch_before": self.t.epoch, "moves": 0, "failed_moves": 0, "rounds": 0,
                       "cutover_s": 0.0, "copy_s": 0.0, "commit_s": 0.0, "bytes": 0}

    def cutover(self) -> None:
        self.t.begin_moves(self.pending)
        self.report["cutover_s"] = self.ctl.push()
        self.report["epoch_cutover"] = self.t.epoch
        if not self.ctl.peers:
            self.ctl.refresh_peers()

    def _retry(self, m: Move, err) -> Optional[Move]:
        """The move to try next round for a failed one (None: give it up)."""
        log.warning("move %s failed: %s", m, err)
        self.report["failed_moves"] += 1
        if m.src is not None:
            src_rank = self.t.rank_of(m.src)
            if src_rank in self.ctl.peers and "unreachable" in str(err):
                self.t.mark_down(src_rank)
        if not self.t.live(self.t.rank_of(m.dst)):
            self.t.finish_moves([m], ok=False)
            return None
        src = self.t.best_source(m.layer, m.expert, m.dst, None)
        return Move(m.layer, m.expert, m.dst, None if src == m.src else src, m.evicts)

    def copy_round(self) -> None:
        self.report["rounds"] += 1
        t0 = time.perf_counter()
        results = self.ctl.engine.move(self.pending, self.ctl.peers, self.t.slots_per_rank)
        self.report["copy_s"] += time.perf_counter() - t0
        answered = {(m.layer, m.dst) for m, _, _ in results}
        done = [m for m, ok, _ in results if ok]
        failed = [(m, err) for m, ok, err in results if not ok]
        failed += [(m, "no result") for m in self.pending if (m.layer, m.dst) not in answered]
        self.t.finish_moves(done, ok=True)
        self.report["moves"] += len(done)
        self.report["bytes"] += sum(self.ctl.move_bytes(m) for m in done)
        self.pending = [nxt for nxt in (self._retry(m, e) for m, e in failed) if nxt is not None]

    def abandon(self) -> None:
        """Leave the remaining destination slots empty (never leak staging slots)."""
        if self.pending:
            self.t.finish_moves(self.pending, ok=False)
            self.pending = []

    def run(self) -> dict:
        t_start = time.perf_counter()
        self.cutover()
        try:
            while self.pending and self.report["rounds"] < self.ctl.max_rounds:
                self.copy_round()
        except BaseException:
            self.abandon()
            try:
                self.ctl.push()
            except Exception:  # noqa: BLE001
                log.exception("ep %s: push after a failed move round failed", self.report["event"])
            raise
        self.abandon()
        self.report["commit_s"] = self.ctl.push()
        self.report["epoch"] = self.t.epoch
        self.report["uncovered"] = len(self.t.uncovered())
        self.report["total_s"] = time.perf_counter() - t_start
        return self.report


class EPController:
    def __init__(self, table: PlacementTable, engine, min_replicas: int = 1, max_rounds: int = 4):
        self.table = table
        self.engine = engine
        self.min_replicas = min_replicas
        self.max_rounds = max_rounds
        self.lock = threading.RLock()
        self.peers: Dict[int, dict] = {}
        self.history: List[dict] = []
        self._installed: Optional[int] = None      # epoch the engines last applied

    def refresh_peers(self) -> dict:
        self.peers = {int(k): v for k, v in (self.engine.describe() or {}).items()}
        return self.peers

    def push(self, force: bool = False) -> float:
        """Commit pending changes and have the engines apply the view; returns
        the seconds the apply took (0 when there was nothing new)."""
        changed = self.table.pending
        self.table.commit()
        if not (changed or force) and self._installed == self.table.epoch:
            return 0.0
        self._installed = self.table.epoch
        t0 = time.perf_counter()
        if self.engine.apply(self.table.view()) is False:
            raise PlacementError(f"engine rejected epoch {self.table.epoch} as stale (another controller?)")
        return time.perf_counter() - t0

    def move_bytes(self, m: Move) -> int:
        desc = self.peers.get(self.table.rank_of(m.dst))
        return sum(nbytes for _, nbytes in desc["layers"][m.layer]) if desc else 0

    def _reconfigure(self, event: str, moves: List[Move]) -> dict:
        report = _Reconfiguration(self, event, moves).run()
        self.history.append(report)
        return report

    # ----------------------------------------------------------------- events
    def fail_rank(self, rank: int) -> dict:
        with self.lock:
            self.table.mark_down(rank)
            self.peers.pop(rank, None)
            return self.reconcile(f"fail rank {rank}")

    def drain_rank(self, rank: int) -> dict:
        with self.lock:
            self.table.mark_draining(rank)
            return self.reconcile(f"drain rank {rank}", prefer_src_rank=rank)

    def left(self, rank: int) -> dict:
        """A rank left for good: route around it, no repair moves."""
        with self.lock:
            self.table.mark_down(rank)
            self.peers.pop(rank, None)
            return {"event": f"left rank {rank}", "epoch": self.table.epoch, "apply_s": self.push()}

    def join_rank(self, rank: int, slot_map_rows=None) -> dict:
        with self.lock:
            self.table.mark_up(rank, slot_map_rows)
            self.refresh_peers()
            return self.reconcile(f"join rank {rank}")

    def _migration(self, pairs, layers, guard_last: bool) -> List[Move]:
        layers = range(self.table.num_layers) if layers is None else layers
        moves = []
        for expert, dst in pairs:
            for layer in layers:
                held = self.table.slot_map[layer][dst]
                if held == expert:
                    continue
                if guard_last and held >= 0 and len(self.table.replicas(layer, held, live_only=True)) <= 1:
                    raise PlacementError(f"slot {dst} holds the last replica of {held}")
                moves.append(Move(layer, expert, dst, self.table.best_source(layer, expert, dst, None), held))
        return moves

    def migrate(self, expert: int, dst_slot: int, layers=None) -> dict:
        """Copy ``expert`` into ``dst_slot`` on every (or the given) layer; the
        slot may not hold the last live copy of another expert."""
        with self.lock:
            return self._reconfigure(f"migrate e{expert}->slot{dst_slot}",
                                     self._migration([(expert, dst_slot)], layers, guard_last=True))

    def migrate_many(self, pairs, layers=None) -> dict:
        """Several (expert, dst_slot) migrations under one pair of epochs."""
        with self.lock:
            return self._reconfigure(f"migrate {len(pairs)} experts", self._migration(pairs, layers, guard_last=False))

    def reconcile(self, event: str = "reconcile", prefer_src_rank=None) -> dict:
        return self._reconfigure(event, self.table.plan_repair(self.min_replicas, prefer_src_rank=prefer_src_rank))


class LocalEngine:
    """An in-process EP group: one :class:`connex.ep.mover.ExpertStore` per
    rank.  ``forward`` runs a toy MoE layer with the installed routing and
    raises when a token would reach a dead rank or an expert with no
    routable copy."""

    loader = None

    def __init__(self, stores, num_experts: int):
        self.stores = {s.rank: s for s in stores}
        self.num_experts = num_experts
        self.view = None
        self.applied: List[int] = []
        self.dead: set = set()

    def apply(self, view: dict) -> bool:
        if self.view is not None and view["epoch"] <= self.view["epoch"]:
            return False
        self.view = view
        self.applied.append(view["epoch"])
        return True

    def describe(self) -> dict:
        return {r: s.describe() for r, s in self.stores.items() if r not in self.dead}

    def move(self, moves, peers, slots_per_rank, loader=None):
        results = []
        for r, store in self.stores.items():
            if r not in self.dead:
                results += store.apply_moves(moves, peers, slots_per_rank, loader=loader or self.loader)
        return results

    def kill(self, rank: int) -> None:
        self.dead.add(rank)
        transport = self.stores[rank].t
        if transport is not None and hasattr(transport, "kill"):
            transport.kill()

    def expert_weight(self, slot: int, layer: int = 0, param: int = 0):
        S = self.view["slots_per_rank"]
        return self.stores[slot // S].layers[layer][param][slot % S]

    def forward(self, x, topk, layer: int = 0):
        l2p, counts = logical_to_physical(self.view, layer)
        S = self.view["slots_per_rank"]
        out = []
        for i, (row, experts) in enumerate(zip(x, topk)):
            acc = torch.zeros_like(row, dtype=torch.float32)
            for e in map(int, experts):
                if counts[e] == 0:
                    raise RuntimeError(f"expert {e} has no routable replica")
                slot = l2p[e][i % counts[e]]
                rank = slot // S
                if rank in self.dead:
                    raise RuntimeError(f"token routed to dead rank {rank}")
                acc += row.float() @ self.stores[rank].layers[layer][0][slot % S].float()
            out.append(acc)
        return torch.stack(out)

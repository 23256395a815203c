"""EP control plane: owns the placement table and drives engines through epochs.

Every reconfiguration (rank fails / drains / joins, expert migrates) runs
the two-epoch protocol of the reference (``connex/ep/controller.py:36-178``):

    epoch k+1  route away from down/draining ranks and from the destination
               slots of the repair moves          -> engines apply the view
    copy       destination ranks pull expert weights from a live replica
               (the checkpoint loader when none is left); a move whose
               source died is re-planned from another source
    epoch k+2  destination slots routable with their new expert -> apply

Engines apply a view only at a step boundary, so no step mixes placements.
An *engine* handle needs ``apply(view)``, ``describe() -> {rank: desc}`` and
``move(moves, peers, slots_per_rank) -> [(move, ok, err)]``.
:class:`LocalEngine` is the in-process EP group used by tests and demos.
"""
from __future__ import annotations

import logging
import threading
import time

import torch

from connex.ep.placement import DOWN, DRAINING, UP, Move, PlacementError, PlacementTable, logical_to_physical

log = logging.getLogger("connex.ep")


class EPController:
    def __init__(self, table: PlacementTable, engine, min_replicas: int = 1, max_rounds: int = 4):
        self.table = table
        self.engine = engine
        self.min_replicas = min_replicas
        self.max_rounds = max_rounds
        self.lock = threading.RLock()
        self.peers: dict = {}
        self.history: list = []
        self._pushed = None

    def refresh_peers(self) -> dict:
        self.peers = {int(k): v for k, v in (self.engine.describe() or {}).items()}
        return self.peers

    def push(self, force: bool = False) -> float:
        """Commit pending changes and install the view; returns seconds."""
        dirty = self.table._dirty
        self.table.commit()
        if not dirty and not force and self._pushed == self.table.epoch:
            return 0.0
        self._pushed = self.table.epoch
        t0 = time.perf_counter()
        if self.engine.apply(self.table.view()) is False:
            raise PlacementError(f"engine rejected epoch {self.table.epoch} as stale (another controller?)")
        return time.perf_counter() - t0

    # ------------------------------------------------------------ events
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
        with self.lock:
            self.table.mark_down(rank)
            self.peers.pop(rank, None)
            return {"event": f"left rank {rank}", "epoch": self.table.epoch, "apply_s": self.push()}

    def join_rank(self, rank: int, slot_map_rows=None) -> dict:
        with self.lock:
            self.table.mark_up(rank, slot_map_rows)
            self.refresh_peers()
            return self.reconcile(f"join rank {rank}")

    def migrate(self, expert: int, dst_slot: int, layers=None) -> dict:
        with self.lock:
            layers = range(self.table.num_layers) if layers is None else layers
            moves = []
            for l in layers:
                old = self.table.slot_map[l][dst_slot]
                if old == expert:
                    continue
                if old >= 0 and len(self.table.replicas(l, old, live_only=True)) <= 1:
                    raise PlacementError(f"slot {dst_slot} holds the last replica of {old}")
                moves.append(Move(l, expert, dst_slot, self.table._pick_src(l, expert, dst_slot), old))
            return self._run_moves(f"migrate e{expert}->slot{dst_slot}", moves)

    def migrate_many(self, pairs, layers=None) -> dict:
        """Several (expert, dst_slot) migrations under one pair of epochs."""
        with self.lock:
            layers = range(self.table.num_layers) if layers is None else layers
            moves = []
            for expert, dst in pairs:
                for l in layers:
                    old = self.table.slot_map[l][dst]
                    if old == expert:
                        continue
                    moves.append(Move(l, expert, dst, self.table._pick_src(l, expert, dst), old))
            return self._run_moves(f"migrate {len(pairs)} experts", moves)

    # -------------------------------------------------------------- core
    def reconcile(self, event: str = "reconcile", prefer_src_rank=None) -> dict:
        return self._run_moves(event, self.table.plan_repair(self.min_replicas, prefer_src_rank=prefer_src_rank))

    def _run_moves(self, event: str, moves) -> dict:
        rep = {"event": event, "epoch_before": self.table.epoch, "moves": 0, "failed_moves": 0, "rounds": 0,
               "cutover_s": 0.0, "copy_s": 0.0, "commit_s": 0.0, "bytes": 0}
        t_start = time.perf_counter()
        self.table.begin_moves(moves)
        rep["cutover_s"] = self.push()
        rep["epoch_cutover"] = self.table.epoch
        if not self.peers:
            self.refresh_peers()
        pending = list(moves)
        try:
            while pending and rep["rounds"] < self.max_rounds:
                rep["rounds"] += 1
                t0 = time.perf_counter()
                res = self.engine.move(pending, self.peers, self.table.slots_per_rank)
                rep["copy_s"] += time.perf_counter() - t0
                done = [m for m, ok, _ in res if ok]
                failed = [(m, err) for m, ok, err in res if not ok]
                seen = {(m.layer, m.dst) for m, _, _ in res}
                failed += [(m, "no result") for m in pending if (m.layer, m.dst) not in seen]
                self.table.finish_moves(done, ok=True)
                rep["moves"] += len(done)
                rep["bytes"] += sum(self._move_bytes(m) for m in done)
                pending = []
                for m, err in failed:
                    log.warning("move %s failed: %s", m, err)
                    rep["failed_moves"] += 1
                    src_rank = None if m.src is None else self.table.rank_of(m.src)
                    if src_rank is not None and src_rank in self.peers and "unreachable" in str(err):
                        self.table.mark_down(src_rank)
                    if not self.table.live(self.table.rank_of(m.dst)):
                        self.table.finish_moves([m], ok=False)
                        continue
                    src = self.table._pick_src(m.layer, m.expert, m.dst, None)
                    pending.append(Move(m.layer, m.expert, m.dst, None if src == m.src else src, m.evicts))
        except BaseException:
            self.table.finish_moves(pending, ok=False)  # never leak staging slots
            try:
                self.push()
            except Exception:
                log.exception("ep %s: push after a failed move round failed", event)
            raise
        if pending:
            self.table.finish_moves(pending, ok=False)
        rep["commit_s"] = self.push()
        rep["epoch"] = self.table.epoch
        rep["uncovered"] = len(self.table.uncovered())
        rep["total_s"] = time.perf_counter() - t_start
        self.history.append(rep)
        return rep

    def _move_bytes(self, m: Move) -> int:
        d = self.peers.get(self.table.rank_of(m.dst))
        return sum(rb for _, rb in d["layers"][m.layer]) if d else 0


class LocalEngine:
    """In-process EP group: one :class:`ExpertStore` per rank; ``forward``
    runs a toy MoE layer with the installed routing and raises if a token
    reaches a dead or unroutable slot."""

    loader = None

    def __init__(self, stores, num_experts: int):
        self.stores = {s.rank: s for s in stores}
        self.num_experts = num_experts
        self.view = None
        self.applied: list = []
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
        out = []
        for r, s in self.stores.items():
            if r not in self.dead:
                out += s.apply_moves(moves, peers, slots_per_rank, loader=loader or self.loader)
        return out

    def kill(self, rank: int) -> None:
        self.dead.add(rank)
        t = self.stores[rank].t
        if t is not None and hasattr(t, "kill"):
            t.kill()

    def expert_weight(self, slot: int, layer: int = 0, param: int = 0):
        S = self.view["slots_per_rank"]
        return self.stores[slot // S].layers[layer][param][slot % S]

    def forward(self, x, topk, layer: int = 0):
        l2p, cnt = logical_to_physical(self.view, layer)
        S = self.view["slots_per_rank"]
        ys = []
        for i, (row, ids) in enumerate(zip(x, topk)):
            acc = torch.zeros_like(row, dtype=torch.float32)
            for e in ids:
                e = int(e)
                if cnt[e] == 0:
                    raise RuntimeError(f"expert {e} has no routable replica")
                slot = l2p[e][i % cnt[e]]
                r = slot // S
                if r in self.dead:
                    raise RuntimeError(f"token routed to dead rank {r}")
                acc += row.float() @ self.stores[r].layers[layer][0][slot % S].float()
            ys.append(acc)
        return torch.stack(ys)

"""Versioned expert placement table (engine neutral, pure Python).

``num_ranks`` EP ranks x ``slots_per_rank`` physical slots; slot ``p`` lives
on rank ``p // slots_per_rank`` and, per MoE layer, ``slot_map[layer][p]`` is
the logical expert it holds (-1 = empty; several slots = replicas).  Ranks
are ``up``, ``draining`` (still serves experts without an up replica) or
``down``; a slot being overwritten by a weight move is ``staging`` and never
routable.  Every change becomes visible only through :meth:`commit`, which
bumps the epoch; engines apply a :meth:`view` at a step boundary when its
epoch is newer than theirs.  :meth:`plan_repair` restores coverage after a
rank drains or dies (destination: empty slot > most-replicated victim >
a rank without the expert > least loaded; source: same rank > preferred
rank > up).  Same semantics and view format as the reference's
``connex/ep/placement.py:42-362``; :func:`logical_to_physical` produces the
``l2p`` / ``l2p_cnt`` tensors the dispatch kernel routes with.
"""
from __future__ import annotations

import copy
from dataclasses import asdict, dataclass
from typing import Iterable, List, Optional

UP, DRAINING, DOWN = "up", "draining", "down"


@dataclass(frozen=True)
class Move:
    layer: int
    expert: int
    dst: int
    src: Optional[int]
    evicts: int = -1

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "Move":
        return cls(**d)


class PlacementError(RuntimeError):
    pass


class PlacementTable:
    def __init__(self, num_experts: int, num_ranks: int, slots_per_rank: int, slot_map: list,
                 num_layers: Optional[int] = None, epoch: int = 0, rank_state: Optional[dict] = None,
                 active_replicas: Optional[int] = None):
        self.num_experts, self.num_ranks, self.slots_per_rank = int(num_experts), int(num_ranks), int(slots_per_rank)
        if slot_map and not isinstance(slot_map[0], (list, tuple)):
            slot_map = [list(slot_map) for _ in range(num_layers or 1)]
        self.slot_map = [list(map(int, row)) for row in slot_map]
        self.num_layers = len(self.slot_map)
        for row in self.slot_map:
            if len(row) != self.num_slots:
                raise PlacementError(f"slot_map row has {len(row)} slots, want {self.num_slots}")
            if any(e < -1 or e >= self.num_experts for e in row):
                raise PlacementError("slot_map holds an out-of-range expert id")
        self.rank_state = {r: UP for r in range(self.num_ranks)}
        if rank_state:
            self.rank_state.update({int(k): v for k, v in rank_state.items()})
        self.staging: set = set()
        self.active_replicas = active_replicas
        self.epoch = int(epoch)
        self._dirty = False

    # ---------------------------------------------------------- construction
    @classmethod
    def linear(cls, num_experts, num_ranks, slots_per_rank, num_layers=1):
        """Slot p holds expert p; redundant slots hold p mod num_experts."""
        P = num_ranks * slots_per_rank
        if P < num_experts:
            raise PlacementError(f"{P} slots cannot hold {num_experts} experts")
        row = [p if p < num_experts else (p - num_experts) % num_experts for p in range(P)]
        return cls(num_experts, num_ranks, slots_per_rank, [row] * num_layers)

    @classmethod
    def spread(cls, num_experts, num_ranks, slots_per_rank, num_layers=1):
        """Replicas of one expert on distinct ranks where capacity allows."""
        R, S, E = num_ranks, slots_per_rank, num_experts
        if R * S < E:
            raise PlacementError(f"{R * S} slots cannot hold {E} experts")
        free = {r: list(range(r * S, (r + 1) * S)) for r in range(R)}
        row = [-1] * (R * S)
        c = 0
        while any(free.values()):
            placed = False
            for e in range(E):
                for k in range(R):
                    r = (e + c + k) % R
                    if free[r] and e not in row[r * S:(r + 1) * S]:
                        row[free[r].pop(0)] = e
                        placed = True
                        break
            c += 1
            if not placed:
                break
        return cls(E, R, S, [row] * num_layers)

    # -------------------------------------------------------------- geometry
    @property
    def num_slots(self) -> int:
        return self.num_ranks * self.slots_per_rank

    def rank_of(self, slot: int) -> int:
        return slot // self.slots_per_rank

    def local_index(self, slot: int) -> int:
        return slot % self.slots_per_rank

    def rank_slots(self, rank: int):
        return range(rank * self.slots_per_rank, (rank + 1) * self.slots_per_rank)

    # --------------------------------------------------------------- queries
    def live(self, rank: int) -> bool:
        return self.rank_state.get(rank) in (UP, DRAINING)

    def replicas(self, layer: int, expert: int, live_only: bool = False) -> List[int]:
        return [p for p, e in enumerate(self.slot_map[layer]) if e == expert and (layer, p) not in self.staging
                and (not live_only or self.live(self.rank_of(p)))]

    def routable_mask(self, layer: int) -> List[bool]:
        row = self.slot_map[layer]
        on_up = {e for p, e in enumerate(row)
                 if e >= 0 and (layer, p) not in self.staging and self.rank_state[self.rank_of(p)] == UP}
        mask = []
        for p, e in enumerate(row):
            st = self.rank_state[self.rank_of(p)]
            mask.append(e >= 0 and (layer, p) not in self.staging and (st == UP or (st == DRAINING and e not in on_up)))
        if self.active_replicas:
            mask = self._limit_active(row, mask, self.active_replicas)
        return mask

    def _limit_active(self, row, mask, k):
        """At most k routed replicas per expert, spread evenly over ranks."""
        cands: dict = {}
        for p, ok in enumerate(mask):
            if ok:
                cands.setdefault(row[p], []).append(p)
        load = {r: 0 for r in range(self.num_ranks)}
        keep = set()
        for e in sorted(cands, key=lambda e: (len(cands[e]), e)):
            ps = list(cands[e])
            for _ in range(min(k, len(ps))):
                p = min(ps, key=lambda q: (load[self.rank_of(q)], (q + e) % len(row)))
                ps.remove(p)
                keep.add(p)
                load[self.rank_of(p)] += 1
        return [p in keep for p in range(len(row))]

    def routable_replicas(self, layer: int, expert: int) -> List[int]:
        m = self.routable_mask(layer)
        return [p for p, e in enumerate(self.slot_map[layer]) if e == expert and m[p]]

    def uncovered(self) -> list:
        out = []
        for layer in range(self.num_layers):
            m = self.routable_mask(layer)
            have = {e for p, e in enumerate(self.slot_map[layer]) if m[p]}
            out.extend((layer, e) for e in range(self.num_experts) if e not in have)
        return out

    def rank_load(self, layer: int = 0) -> dict:
        m = self.routable_mask(layer)
        load = {r: 0 for r in range(self.num_ranks)}
        for p, ok in enumerate(m):
            if ok:
                load[self.rank_of(p)] += 1
        return load

    # ------------------------------------------------------------- mutations
    def set_rank_state(self, rank: int, state: str) -> None:
        if state not in (UP, DRAINING, DOWN):
            raise ValueError(state)
        if rank >= self.num_ranks:
            raise PlacementError(f"rank {rank} out of range")
        if self.rank_state[rank] != state:
            self.rank_state[rank] = state
            if state == DOWN:
                self.staging = {(l, p) for l, p in self.staging if self.rank_of(p) != rank}
            self._dirty = True

    def mark_down(self, rank: int) -> None:
        self.set_rank_state(rank, DOWN)

    def mark_draining(self, rank: int) -> None:
        self.set_rank_state(rank, DRAINING)

    def mark_up(self, rank: int, slot_map_rows=None) -> None:
        if slot_map_rows is not None:
            for layer, row in enumerate(slot_map_rows):
                for i, e in enumerate(row):
                    self.slot_map[layer][rank * self.slots_per_rank + i] = int(e)
        self.set_rank_state(rank, UP)

    def begin_moves(self, moves: Iterable[Move]) -> None:
        for m in moves:
            if not self.live(self.rank_of(m.dst)):
                raise PlacementError(f"move to slot {m.dst} on a dead rank")
            self.staging.add((m.layer, m.dst))
        self._dirty = True

    def finish_moves(self, moves: Iterable[Move], ok: bool = True) -> None:
        for m in moves:
            self.staging.discard((m.layer, m.dst))
            if self.live(self.rank_of(m.dst)):
                self.slot_map[m.layer][m.dst] = m.expert if ok else -1
        self._dirty = True

    def commit(self) -> int:
        if self._dirty:
            self.epoch += 1
            self._dirty = False
        return self.epoch

    # -------------------------------------------------------------- planning
    def plan_repair(self, min_replicas: int = 1, prefer_src_rank: Optional[int] = None) -> List[Move]:
        moves = []
        for layer in range(self.num_layers):
            row = self.slot_map[layer]
            reserved: set = set()
            up_reps = {e: [p for p, x in enumerate(row) if x == e and (layer, p) not in self.staging
                           and self.rank_state[self.rank_of(p)] == UP] for e in range(self.num_experts)}
            for e in sorted((e for e in range(self.num_experts) if len(up_reps[e]) < min_replicas),
                            key=lambda e: len(up_reps[e])):
                while len(up_reps[e]) < min_replicas:
                    dst = self._pick_dst(layer, e, up_reps, reserved)
                    if dst is None:
                        break
                    src = self._pick_src(layer, e, dst, prefer_src_rank)
                    old = row[dst]
                    if old >= 0 and dst in up_reps.get(old, []):
                        up_reps[old].remove(dst)
                    reserved.add(dst)
                    up_reps[e].append(dst)
                    moves.append(Move(layer, e, dst, src, old))
        return moves

    def _pick_dst(self, layer, expert, up_reps, reserved):
        row = self.slot_map[layer]
        load = {r: 0 for r in range(self.num_ranks)}
        for p, x in enumerate(row):
            if x >= 0:
                load[self.rank_of(p)] += 1
        have_rank = {self.rank_of(p) for p in up_reps[expert]}
        best, best_key = None, None
        for p, x in enumerate(row):
            r = self.rank_of(p)
            if self.rank_state[r] != UP or p in reserved or (layer, p) in self.staging or x == expert:
                continue
            if x >= 0 and len(up_reps.get(x, [])) <= 1:
                continue  # would strand the expert it holds
            key = (x >= 0, -len(up_reps.get(x, [])) if x >= 0 else 0, r in have_rank, load[r], p)
            if best_key is None or key < best_key:
                best, best_key = p, key
        return best

    def _pick_src(self, layer, expert, dst, prefer_rank=None):
        cands = [p for p, x in enumerate(self.slot_map[layer]) if x == expert and (layer, p) not in self.staging
                 and self.live(self.rank_of(p)) and p != dst]
        if not cands:
            return None
        dr = self.rank_of(dst)
        return min(cands, key=lambda p: (self.rank_of(p) != dr, prefer_rank is not None and self.rank_of(p) != prefer_rank,
                                         self.rank_state[self.rank_of(p)] != UP, p))

    # ---------------------------------------------------------- serialising
    def view(self) -> dict:
        return {"epoch": self.epoch, "num_experts": self.num_experts, "num_ranks": self.num_ranks,
                "slots_per_rank": self.slots_per_rank, "slot_map": copy.deepcopy(self.slot_map),
                "routable": [self.routable_mask(l) for l in range(self.num_layers)],
                "rank_state": {str(r): s for r, s in self.rank_state.items()},
                "active_replicas": self.active_replicas}

    def to_dict(self) -> dict:
        d = self.view()
        d["staging"] = sorted(self.staging)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "PlacementTable":
        t = cls(d["num_experts"], d["num_ranks"], d["slots_per_rank"], d["slot_map"], epoch=d.get("epoch", 0),
                rank_state=d.get("rank_state"), active_replicas=d.get("active_replicas"))
        t.staging = {tuple(x) for x in d.get("staging", [])}
        return t


def logical_to_physical(view: dict, layer: int, max_replicas: Optional[int] = None):
    """``(l2p, counts)`` of one layer: routable slots per logical expert padded
    with -1 to ``max_replicas``, and replica counts."""
    row, mask = view["slot_map"][layer], view["routable"][layer]
    l2p: List[list] = [[] for _ in range(view["num_experts"])]
    for p, (e, ok) in enumerate(zip(row, mask)):
        if ok and e >= 0:
            l2p[e].append(p)
    width = max_replicas or max(1, max(len(x) for x in l2p))
    counts = [len(x) for x in l2p]
    if max(counts) > width:
        raise PlacementError(f"an expert has {max(counts)} replicas, engine allows {width}")
    return [x + [-1] * (width - len(x)) for x in l2p], counts


def l2p_tensors(view: dict, layer: int, device, max_replicas: Optional[int] = None):
    """The ``l2p [E, R]`` / ``l2p_cnt [E]`` int32 device tensors of a layer."""
    import torch
    l2p, counts = logical_to_physical(view, layer, max_replicas)
    return (torch.tensor(l2p, dtype=torch.int32, device=device),
            torch.tensor(counts, dtype=torch.int32, device=device))

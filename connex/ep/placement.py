"""Versioned expert placement table (engine neutral, pure Python).

Geometry: ``num_ranks`` EP ranks with ``slots_per_rank`` physical expert
slots each; slot ``p`` lives on rank ``p // slots_per_rank``.  Per MoE layer
``slot_map[layer][p]`` is the logical expert slot ``p`` holds (-1 = empty;
an expert in several slots has replicas).

Routing rules (:meth:`PlacementTable.routable_mask`):

* a slot in ``staging`` (being overwritten by a weight move) never routes;
* slots on an ``up`` rank route;
* a ``draining`` rank routes only experts that have no replica on an up rank;
* a ``down`` rank routes nothing;
* with ``active_replicas = k`` at most k replicas of an expert route, chosen
  to balance the routed slots per rank (the others are warm standbys).

Nothing becomes visible until :meth:`commit` bumps the epoch; engines apply
a :meth:`view` at a step boundary when its epoch is newer than theirs.
:meth:`plan_repair` restores ``min_replicas`` up copies of every expert:
destinations score empty slots first, then the slot of the most replicated
other expert (never the last up copy of anything), then ranks that lack the
expert, then the least loaded rank; sources score the destination's own
rank first, then a preferred rank, then up ranks over draining ones.

Semantics and the view format follow ``connex/ep/placement.py:42-362`` of
the reference; :func:`logical_to_physical` yields the ``l2p`` / ``l2p_cnt``
maps the EP dispatch kernel routes with.
"""
from __future__ import annotations

import copy
import heapq
from dataclasses import asdict, dataclass
from typing import Dict, Iterable, List, Optional, Set, Tuple

UP, DRAINING, DOWN = "up", "draining", "down"
_STATES = (UP, DRAINING, DOWN)


@dataclass(frozen=True)
class Move:
    """Copy ``expert``'s weights of ``layer`` into slot ``dst`` (from slot
    ``src``, or from the checkpoint when None); ``evicts`` is the expert the
    slot held before (-1 = empty)."""

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
        self.num_experts, self.num_ranks = int(num_experts), int(num_ranks)
        self.slots_per_rank = int(slots_per_rank)
        flat = bool(slot_map) and not isinstance(slot_map[0], (list, tuple))
        rows = [list(slot_map)] * (num_layers or 1) if flat else slot_map
        self.slot_map: List[List[int]] = [[int(e) for e in row] for row in rows]
        self.num_layers = len(self.slot_map)
        self._validate()
        self.rank_state: Dict[int, str] = dict.fromkeys(range(self.num_ranks), UP)
        self.rank_state.update({int(k): v for k, v in (rank_state or {}).items()})
        self.staging: Set[Tuple[int, int]] = set()
        self.active_replicas = active_replicas
        self.epoch = int(epoch)
        self._dirty = False

    def _validate(self) -> None:
        for row in self.slot_map:
            if len(row) != self.num_slots:
                raise PlacementError(f"slot_map row has {len(row)} slots, want {self.num_slots}")
            if not all(-1 <= e < self.num_experts for e in row):
                raise PlacementError("slot_map holds an out-of-range expert id")

    # --------------------------------------------------------- constructions
    @classmethod
    def linear(cls, num_experts, num_ranks, slots_per_rank, num_layers=1):
        """Slot p holds expert p; slots beyond the experts hold replicas in order."""
        slots = num_ranks * slots_per_rank
        if slots < num_experts:
            raise PlacementError(f"{slots} slots cannot hold {num_experts} experts")
        row = [p % num_experts for p in range(slots)]
        return cls(num_experts, num_ranks, slots_per_rank, [row] * num_layers)

    @classmethod
    def spread(cls, num_experts, num_ranks, slots_per_rank, num_layers=1):
        """Copies handed out expert by expert, round after round, each copy to
        the next rank (from a per-expert rotating start) with a free slot that
        does not hold the expert yet; a copy that fits nowhere is skipped."""
        R, S, E = num_ranks, slots_per_rank, num_experts
        if R * S < E:
            raise PlacementError(f"{R * S} slots cannot hold {E} experts")
        holds: List[List[int]] = [[] for _ in range(R)]
        for rnd in range(R * S):
            placed = 0
            for e in range(E):
                for k in range(R):
                    r = (e + rnd + k) % R
                    if len(holds[r]) < S and e not in holds[r]:
                        holds[r].append(e)
                        placed += 1
                        break
            if placed == 0 or all(len(h) == S for h in holds):
                break
        row = [e for h in holds for e in h + [-1] * (S - len(h))]
        return cls(E, R, S, [row] * num_layers)

    # --------------------------------------------------------------- geometry
    @property
    def num_slots(self) -> int:
        return self.num_ranks * self.slots_per_rank

    def rank_of(self, slot: int) -> int:
        return slot // self.slots_per_rank

    def local_index(self, slot: int) -> int:
        return slot % self.slots_per_rank

    def rank_slots(self, rank: int):
        return range(rank * self.slots_per_rank, (rank + 1) * self.slots_per_rank)

    # ---------------------------------------------------------------- queries
    def _state_of(self, slot: int) -> str:
        return self.rank_state[self.rank_of(slot)]

    def live(self, rank: int) -> bool:
        return self.rank_state.get(rank) in (UP, DRAINING)

    def _usable(self, layer: int, slot: int) -> bool:
        return self.slot_map[layer][slot] >= 0 and (layer, slot) not in self.staging

    def replicas(self, layer: int, expert: int, live_only: bool = False) -> List[int]:
        return [p for p, e in enumerate(self.slot_map[layer])
                if e == expert and (layer, p) not in self.staging and (not live_only or self.live(self.rank_of(p)))]

    def _up_copies(self, layer: int) -> Dict[int, List[int]]:
        """expert -> its usable slots on up ranks."""
        out: Dict[int, List[int]] = {e: [] for e in range(self.num_experts)}
        for p, e in enumerate(self.slot_map[layer]):
            if self._usable(layer, p) and self._state_of(p) == UP:
                out[e].append(p)
        return out

    def routable_mask(self, layer: int) -> List[bool]:
        up = self._up_copies(layer)
        mask = []
        for p, e in enumerate(self.slot_map[layer]):
            state = self._state_of(p)
            serves = state == UP or (state == DRAINING and not up.get(e))
            mask.append(self._usable(layer, p) and serves)
        if self.active_replicas:
            mask = self._limit_active(self.slot_map[layer], mask, self.active_replicas)
        return mask

    def _limit_active(self, row, mask, k):
        """Keep at most ``k`` routed copies per expert.  Experts with the fewest
        candidates choose first; each takes, one copy at a time, the candidate
        on the rank with the fewest kept copies so far (ties by a rotation of
        the slot index by the expert id, so experts do not all favour slot 0)."""
        by_expert: Dict[int, List[int]] = {}
        for p, ok in enumerate(mask):
            if ok:
                by_expert.setdefault(row[p], []).append(p)
        kept_per_rank = [0] * self.num_ranks
        keep: Set[int] = set()
        for e in sorted(by_expert, key=lambda x: (len(by_expert[x]), x)):
            heap = [(kept_per_rank[self.rank_of(p)], (p + e) % len(row), p) for p in by_expert[e]]
            for _ in range(min(k, len(heap))):
                heapq.heapify(heap)                 # loads changed since the last pick
                _, _, p = heapq.heappop(heap)
                keep.add(p)
                kept_per_rank[self.rank_of(p)] += 1
                heap = [(kept_per_rank[self.rank_of(q)], t, q) for _, t, q in heap]
        return [p in keep for p in range(len(row))]

    def routable_replicas(self, layer: int, expert: int) -> List[int]:
        mask = self.routable_mask(layer)
        return [p for p, e in enumerate(self.slot_map[layer]) if e == expert and mask[p]]

    def uncovered(self) -> list:
        """(layer, expert) pairs no slot routes."""
        gaps = []
        for layer in range(self.num_layers):
            mask = self.routable_mask(layer)
            routed = {e for e, ok in zip(self.slot_map[layer], mask) if ok}
            gaps += [(layer, e) for e in range(self.num_experts) if e not in routed]
        return gaps

    def rank_load(self, layer: int = 0) -> dict:
        load = dict.fromkeys(range(self.num_ranks), 0)
        for p, ok in enumerate(self.routable_mask(layer)):
            load[self.rank_of(p)] += ok
        return load

    # -------------------------------------------------------------- mutations
    def set_rank_state(self, rank: int, state: str) -> None:
        if state not in _STATES:
            raise ValueError(state)
        if rank >= self.num_ranks:
            raise PlacementError(f"rank {rank} out of range")
        if self.rank_state[rank] == state:
            return
        self.rank_state[rank] = state
        if state == DOWN:      # moves into a dead rank's slots are void
            self.staging = {(l, p) for l, p in self.staging if self.rank_of(p) != rank}
        self._dirty = True

    def mark_down(self, rank: int) -> None:
        self.set_rank_state(rank, DOWN)

    def mark_draining(self, rank: int) -> None:
        self.set_rank_state(rank, DRAINING)

    def mark_up(self, rank: int, slot_map_rows=None) -> None:
        """Bring a rank (back) up; ``slot_map_rows[layer]`` (optional) are the
        experts its slots hold now."""
        for layer, row in enumerate(slot_map_rows or ()):
            first = rank * self.slots_per_rank
            self.slot_map[layer][first:first + len(row)] = [int(e) for e in row]
        self.set_rank_state(rank, UP)

    def begin_moves(self, moves: Iterable[Move]) -> None:
        moves = list(moves)
        dead = [m.dst for m in moves if not self.live(self.rank_of(m.dst))]
        if dead:
            raise PlacementError(f"move to slot {dead[0]} on a dead rank")
        self.staging.update((m.layer, m.dst) for m in moves)
        self._dirty = True

    def finish_moves(self, moves: Iterable[Move], ok: bool = True) -> None:
        for m in moves:
            self.staging.discard((m.layer, m.dst))
            if self.live(self.rank_of(m.dst)):
                self.slot_map[m.layer][m.dst] = m.expert if ok else -1
        self._dirty = True

    @property
    def pending(self) -> bool:
        """Changes made since the last commit."""
        return self._dirty

    def commit(self) -> int:
        """Publish the pending changes as a new epoch (no bump when clean)."""
        self.epoch += self._dirty
        self._dirty = False
        return self.epoch

    # --------------------------------------------------------------- planning
    def plan_repair(self, min_replicas: int = 1, prefer_src_rank: Optional[int] = None) -> List[Move]:
        """Moves that give every expert ``min_replicas`` copies on up ranks
        (best effort: no move takes the last up copy of another expert)."""
        plan: List[Move] = []
        for layer in range(self.num_layers):
            copies = self._up_copies(layer)
            taken: Set[int] = set()
            short = [e for e in range(self.num_experts) if len(copies[e]) < min_replicas]
            for e in sorted(short, key=lambda x: len(copies[x])):
                while len(copies[e]) < min_replicas:
                    dst = self._best_destination(layer, e, copies, taken)
                    if dst is None:
                        break
                    victim = self.slot_map[layer][dst]
                    if victim >= 0 and dst in copies.get(victim, ()):
                        copies[victim].remove(dst)
                    taken.add(dst)
                    copies[e].append(dst)
                    plan.append(Move(layer, e, dst, self.best_source(layer, e, dst, prefer_src_rank), victim))
        return plan

    def _best_destination(self, layer: int, expert: int, copies: Dict[int, List[int]], taken: Set[int]):
        row = self.slot_map[layer]
        filled = [0] * self.num_ranks
        for p, x in enumerate(row):
            filled[self.rank_of(p)] += x >= 0
        has_it = {self.rank_of(p) for p in copies[expert]}

        def score(p: int):
            x, r = row[p], self.rank_of(p)
            return (x >= 0, -len(copies.get(x, ())) if x >= 0 else 0, r in has_it, filled[r], p)

        options = [p for p, x in enumerate(row)
                   if self._state_of(p) == UP and p not in taken and (layer, p) not in self.staging and x != expert
                   and not (x >= 0 and len(copies.get(x, ())) <= 1)]
        return min(options, key=score) if options else None

    def best_source(self, layer: int, expert: int, dst: int, prefer_rank: Optional[int] = None):
        options = [p for p, x in enumerate(self.slot_map[layer])
                   if x == expert and p != dst and (layer, p) not in self.staging and self.live(self.rank_of(p))]
        if not options:
            return None

        def score(p: int):
            r = self.rank_of(p)
            return r != self.rank_of(dst), prefer_rank is not None and r != prefer_rank, self.rank_state[r] != UP, p

        return min(options, key=score)

    # ------------------------------------------------------------ serialising
    def view(self) -> dict:
        return {"epoch": self.epoch, "num_experts": self.num_experts, "num_ranks": self.num_ranks,
                "slots_per_rank": self.slots_per_rank, "slot_map": copy.deepcopy(self.slot_map),
                "routable": [self.routable_mask(l) for l in range(self.num_layers)],
                "rank_state": {str(r): s for r, s in self.rank_state.items()},
                "active_replicas": self.active_replicas}

    def to_dict(self) -> dict:
        return {**self.view(), "staging": sorted(self.staging)}

    @classmethod
    def from_dict(cls, d: dict) -> "PlacementTable":
        t = cls(d["num_experts"], d["num_ranks"], d["slots_per_rank"], d["slot_map"], epoch=d.get("epoch", 0),
                rank_state=d.get("rank_state"), active_replicas=d.get("active_replicas"))
        t.staging = {tuple(x) for x in d.get("staging", [])}
        return t


def logical_to_physical(view: dict, layer: int, max_replicas: Optional[int] = None):
    """``(l2p, counts)`` of one layer of a view: per logical expert the
    routable slots padded with -1 to ``max_replicas`` (default: the largest
    replica count), and the replica counts."""
    routed: List[List[int]] = [[] for _ in range(view["num_experts"])]
    for p, (e, ok) in enumerate(zip(view["slot_map"][layer], view["routable"][layer])):
        if ok and e >= 0:
            routed[e].append(p)
    counts = [len(x) for x in routed]
    width = max_replicas or max(1, max(counts))
    if max(counts) > width:
        raise PlacementError(f"an expert has {max(counts)} replicas, engine allows {width}")
    return [x + [-1] * (width - len(x)) for x in routed], counts


def l2p_tensors(view: dict, layer: int, device, max_replicas: Optional[int] = None):
    """The ``l2p [E, R]`` / ``l2p_cnt [E]`` int32 device tensors of a layer."""
    import torch
    l2p, counts = logical_to_physical(view, layer, max_replicas)
    return (torch.tensor(l2p, dtype=torch.int32, device=device),
            torch.tensor(counts, dtype=torch.int32, device=device))

"""Sticky peer selection for a pipeline stage, and an in-process membership.

``select_peer`` rules, in order (reference ``connex/pp/routing.py:49-109``):
drop addresses listed under more than one stage (stale artefacts; fall back
to the unfiltered list if that empties it), drop ``exclude_replica``, skip
departed replicas unless nothing else is left, keep ``current`` if still
listed, else the only one, else rank based (``my_rank % n`` over the sorted
replicas of my own stage).
"""
from __future__ import annotations

import logging
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Callable, Iterable, Optional

_log = logging.getLogger("connex.pp.routing")


@dataclass(frozen=True)
class Lid:
    stage_idx: int
    replica_idx: int
    model_name: str = "default"


@dataclass
class Route:
    lid: Lid
    addresses: list = field(default_factory=list)


def select_peer(all_peers: list, target_stage: int, my_stage: int, my_replica: int, current: Optional[int],
                deregistered: set, exclude_replica: Optional[int] = None, log: logging.Logger = _log):
    """-> (address, replica_idx, is_new_choice) or (None, None, False)."""
    stages_of: dict = defaultdict(set)
    for r in all_peers:
        for a in r.addresses:
            stages_of[a].add(r.lid.stage_idx)
    ambiguous = {a for a, st in stages_of.items() if len(st) > 1}

    def cands(skip_ambiguous: bool):
        return [r for r in all_peers
                if r.lid.stage_idx == target_stage and r.addresses
                and not (skip_ambiguous and r.addresses[0] in ambiguous)
                and (exclude_replica is None or r.lid.replica_idx != exclude_replica)]

    peers = cands(True) or cands(False)
    if ambiguous:
        log.warning("stage %s: ignoring addresses listed under several stages: %s", my_stage, sorted(ambiguous))
    live = [r for r in peers if (r.lid.stage_idx, r.lid.replica_idx) not in deregistered]
    peers = live or peers
    if not peers:
        return None, None, False
    for r in peers:
        if r.lid.replica_idx == current:
            return r.addresses[0], current, False
    if len(peers) == 1:
        return peers[0].addresses[0], peers[0].lid.replica_idx, True
    mine = sorted((r for r in all_peers if r.lid.stage_idx == my_stage and r.addresses),
                  key=lambda r: r.lid.replica_idx)
    my_rank = next((i for i, p in enumerate(mine) if p.lid.replica_idx == my_replica), 0)
    peers = sorted(peers, key=lambda r: r.lid.replica_idx)
    sel = peers[my_rank % len(peers)]
    return sel.addresses[0], sel.lid.replica_idx, True


class StaticMembership:
    """In-process membership with the EPC client's duck type (tests, fixed
    deployments); ``emit`` delivers events shaped like the EPC client's."""

    def __init__(self, stage_idx: int, replica_idx: int = 0, routes: Iterable = (), model_name: str = "default"):
        self.lid = Lid(stage_idx, replica_idx, model_name)
        self.routes: list = list(routes)
        self.refreshes = 0
        self._handlers: dict = defaultdict(list)

    def start(self) -> bool:
        return True

    def stop(self) -> None:
        pass

    def refresh_routes(self) -> None:
        self.refreshes += 1

    def get_pipeline_peers(self) -> list:
        return list(self.routes)

    def get_stage_peers(self, stage_idx: int, refresh: str = "auto") -> list:
        if refresh == "always":
            self.refreshes += 1
        return [r for r in self.routes if r.lid.stage_idx == stage_idx]

    def on_event(self, event_type, callback: Callable) -> None:
        self._handlers[event_type].append(callback)

    def add(self, stage_idx: int, replica_idx: int, address: str) -> Route:
        r = Route(Lid(stage_idx, replica_idx), [address])
        self.routes.append(r)
        return r

    def remove(self, stage_idx: int, replica_idx: int) -> None:
        self.routes = [r for r in self.routes if (r.lid.stage_idx, r.lid.replica_idx) != (stage_idx, replica_idx)]

    def emit(self, event_type, stage_idx: int, replica_idx: int, **payload) -> None:
        ev = type("MembershipEvent", (), {})()
        ev.payload = {"lid": {"stage_idx": stage_idx, "replica_idx": replica_idx}, **payload}
        for cb in list(self._handlers.get(event_type, ())):
            cb(ev)

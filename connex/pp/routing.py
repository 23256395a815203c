"""Sticky choice of the next-stage replica, and an in-process membership.

:func:`select_peer` narrows the routes of the target stage step by step and
then picks one:

1. addresses that the membership lists under more than one stage are
   stale artefacts of a migration and are ignored -- unless that would leave
   nothing, in which case the unfiltered routes are used;
2. ``exclude_replica`` (the replica being failed away from) is removed;
3. replicas known to have departed are skipped while any other is left;
4. the replica in use (``current``) is kept if it is still a candidate;
5. otherwise a lone candidate is taken, and with several the sender's rank
   among its own stage's replicas, modulo the number of candidates, spreads
   the senders over the receivers deterministically.

Behavioural parity: ``connex/pp/routing.py:49-161`` of the reference.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Set, Tuple

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

    @property
    def key(self) -> Tuple[int, int]:
        return self.lid.stage_idx, self.lid.replica_idx

    @property
    def address(self) -> Optional[str]:
        return self.addresses[0] if self.addresses else None


def _shared_addresses(routes: List[Route]) -> Set[str]:
    """Addresses that appear under two or more stages."""
    owner: Dict[str, int] = {}
    shared: Set[str] = set()
    for r in routes:
        for a in r.addresses:
            if owner.setdefault(a, r.lid.stage_idx) != r.lid.stage_idx:
                shared.add(a)
    return shared


def _sender_rank(routes: List[Route], stage: int, replica: int) -> int:
    """Position of (stage, replica) among that stage's addressed replicas, by index."""
    mine = sorted(r.lid.replica_idx for r in routes if r.lid.stage_idx == stage and r.addresses)
    return mine.index(replica) if replica in mine else 0


def select_peer(all_peers: list, target_stage: int, my_stage: int, my_replica: int, current: Optional[int],
                deregistered: set, exclude_replica: Optional[int] = None, log: logging.Logger = _log):
    """Returns ``(address, replica_idx, is_new_choice)``, or ``(None, None, False)``
    when the target stage has no usable replica."""
    target = [r for r in all_peers if r.lid.stage_idx == target_stage and r.addresses
              and r.lid.replica_idx != exclude_replica]
    shared = _shared_addresses(all_peers)
    if shared:
        log.warning("stage %s: ignoring addresses listed under several stages: %s", my_stage, sorted(shared))
        target = [r for r in target if r.address not in shared] or target
    present = [r for r in target if r.key not in deregistered]
    target = present or target
    if not target:
        return None, None, False
    keep = next((r for r in target if r.lid.replica_idx == current), None)
    if keep is not None:
        return keep.address, current, False
    if len(target) == 1:
        choice = target[0]
    else:
        target.sort(key=lambda r: r.lid.replica_idx)
        choice = target[_sender_rank(all_peers, my_stage, my_replica) % len(target)]
    return choice.address, choice.lid.replica_idx, True


class _Event:
    """An event object shaped like the EPC client's (``.payload`` dict)."""

    def __init__(self, payload: dict):
        self.payload = payload


class StaticMembership:
    """In-process membership with the EPC client's duck type, for tests and
    fixed deployments: routes are added and removed by hand and ``emit``
    delivers an event to the handlers registered for its type."""

    def __init__(self, stage_idx: int, replica_idx: int = 0, routes: Iterable = (), model_name: str = "default"):
        self.lid = Lid(stage_idx, replica_idx, model_name)
        self.routes: List[Route] = list(routes)
        self.refreshes = 0
        self._handlers: Dict[object, List[Callable]] = {}

    def start(self) -> bool:
        return True

    def stop(self) -> None:
        pass

    def refresh_routes(self) -> None:
        self.refreshes += 1

    def get_pipeline_peers(self) -> list:
        return list(self.routes)

    def get_stage_peers(self, stage_idx: int, refresh: str = "auto") -> list:
        self.refreshes += refresh == "always"
        return [r for r in self.routes if r.lid.stage_idx == stage_idx]

    def on_event(self, event_type, callback: Callable) -> None:
        self._handlers.setdefault(event_type, []).append(callback)

    def add(self, stage_idx: int, replica_idx: int, address: str) -> Route:
        route = Route(Lid(stage_idx, replica_idx), [address])
        self.routes.append(route)
        return route

    def remove(self, stage_idx: int, replica_idx: int) -> None:
        self.routes = [r for r in self.routes if r.key != (stage_idx, replica_idx)]

    def emit(self, event_type, stage_idx: int, replica_idx: int, **payload) -> None:
        ev = _Event({"lid": {"stage_idx": stage_idx, "replica_idx": replica_idx}, **payload})
        for cb in list(self._handlers.get(event_type, ())):
            cb(ev)

"""Transport peer-death events -> group failure reports.

A transfer engine reports link events as dicts ``{"type": "up" | "joined" |
"failed", "peer": (model, stage, shard, replica), "reason": str}``.  A TP
group is one endpoint, so the death of any rank must fail the whole group at
the front router, once, and only for real deaths.

:class:`GroupFailureTracker` is that policy as a small state machine per
peer identity (only identities of the watched model and stages count):

============  ==============================  ==================
state         event                           result
============  ==============================  ==================
(any)         ``up`` / ``joined``             -> LINKED
LINKED        ``failed``, reason not timeout  -> REPORTED, report
LINKED        ``failed``, reason timeout      stays (suspicion only;
                                              the lease decides)
unknown /     ``failed``                      ignored (the link was
REPORTED                                      never up, or already
                                              reported this incarnation)
============  ==============================  ==================

:class:`EventPump` reads ``engine.wait_event`` on a thread and hands every
event to a callback; :class:`PeerDeathReporter` combines the two and
reports dead peers to the front router (which fails their group).  The PP
endpoint and the EP group watcher use the same pump.
Behavioural parity: ``connex/pd/group.py:39-179`` of the reference.
"""
from __future__ import annotations

import logging
import threading
import time
from typing import Callable, Dict, Iterable, List, Optional, Tuple

from connex.protocol import LogicalEndpointID

log = logging.getLogger("connex.pd")

LINKED, REPORTED = "linked", "reported"
PeerKey = Tuple[str, int, int, int]


def peer_key(ev: dict) -> Optional[PeerKey]:
    """The (model, stage, shard, replica) an engine event names, or None."""
    peer = ev.get("peer")
    if not peer or len(peer) < 4:
        return None
    try:
        return str(peer[0]), int(peer[1]), int(peer[2]), int(peer[3])
    except (TypeError, ValueError):
        return None


def is_timeout(ev: dict) -> bool:
    return "timeout" in str(ev.get("reason", ""))


class GroupFailureTracker:
    def __init__(self, model: Optional[str], stages: Iterable[int]):
        self.model = model
        self.stages = frozenset(int(s) for s in stages)
        self.state: Dict[PeerKey, str] = {}

    # views kept for callers that inspect the tracker
    @property
    def up(self) -> set:
        return {k for k, s in self.state.items() if s == LINKED}

    @property
    def reported(self) -> set:
        return {k for k, s in self.state.items() if s == REPORTED}

    def _watched(self, key: PeerKey) -> bool:
        return key[1] in self.stages and (not self.model or key[0] == self.model)

    def on_event(self, ev: dict) -> Optional[LogicalEndpointID]:
        """The LID to report for this event, or None."""
        key = peer_key(ev)
        if key is None or not self._watched(key):
            return None
        kind = ev.get("type")
        if kind in ("up", "joined"):
            self.state[key] = LINKED
            return None
        if kind == "failed" and self.state.get(key) == LINKED and not is_timeout(ev):
            self.state[key] = REPORTED
            return LogicalEndpointID(*key)
        return None


class EventPump:
    """Reads ``engine.wait_event(poll_ms)`` on a daemon thread and calls
    ``handler(event)`` for each; ends on :meth:`stop` or when the engine
    raises (closed)."""

    def __init__(self, engine, handler: Callable[[dict], object], name: str = "connex-peer-watch",
                 poll_ms: int = 100):
        self.engine, self.handler, self.poll_ms = engine, handler, poll_ms
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name=name, daemon=True)

    def start(self) -> "EventPump":
        self._thread.start()
        return self

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                ev = self.engine.wait_event(self.poll_ms)
            except Exception:  # noqa: BLE001 - the engine was closed
                return
            if ev is None:
                continue
            try:
                self.handler(ev)
            except Exception:  # noqa: BLE001 - a failing handler must not end the watch
                log.exception("peer event handler")

    def stop(self) -> None:
        self._stop.set()


class PeerDeathReporter:
    """Reports each confirmed peer death to the front router once.
    ``resolve(lid)`` (optional) maps an engine identity to the PD member it
    belongs to (None: not one of ours)."""

    def __init__(self, engine, front_router_api: str, model: Optional[str], stages: Optional[Iterable[int]] = None,
                 report: Optional[Callable[[LogicalEndpointID, str], object]] = None,
                 resolve: Optional[Callable[[LogicalEndpointID], Optional[LogicalEndpointID]]] = None):
        if stages is None:
            from connex.pd.membership import PD_STAGE
            stages = PD_STAGE.values()
        self.engine = engine
        self.front_router = front_router_api
        self.tracker = GroupFailureTracker(model, stages)
        self._report = report if report is not None else self._report_to_router
        self._resolve = resolve
        self._pump = EventPump(engine, self.handle, name="connex-pd-peer-watch")
        self.reports: List[tuple] = []

    def _report_to_router(self, lid: LogicalEndpointID, reason: str):
        from connex.pd.membership import report_failure
        return report_failure(self.front_router, lid, reason)

    def start(self) -> None:
        self._pump.start()

    def stop(self) -> None:
        self._pump.stop()

    def _member_of(self, lid: LogicalEndpointID) -> Optional[LogicalEndpointID]:
        if self._resolve is None:
            return lid
        try:
            return self._resolve(lid)
        except Exception:  # noqa: BLE001 - unresolvable: not reported
            return None

    def handle(self, ev: dict) -> Optional[LogicalEndpointID]:
        lid = self.tracker.on_event(ev)
        lid = self._member_of(lid) if lid is not None else None
        if lid is None:
            return None
        log.warning("%s rank %d of replica %d died: reporting its group", lid.model_name, lid.shard_idx,
                    lid.replica_idx)
        try:
            outcome = self._report(lid, f"peer died ({ev.get('reason', 'transport event')})")
        except Exception as e:  # noqa: BLE001 - recorded, the watch goes on
            outcome = e
        self.reports.append((time.time(), lid, outcome))
        return lid


def rs_port_resolver(front_router_api: str, model: str, timeout_ms: int = 1000):
    """Resolver for engines that name a peer by its engine port
    (``(model, stage, 0, port)``): the PD member whose addresses include
    ``rs=host:<port>``, if exactly one does."""
    from connex.pd.membership import PD_STAGE, _router_call

    def resolve(lid: LogicalEndpointID) -> Optional[LogicalEndpointID]:
        rep = _router_call(front_router_api, "get_routes",
                           {"model_name": model, "stage_idx": list(PD_STAGE.values()), "compact": True}, timeout_ms)
        if rep is None:
            return None
        suffix = f":{lid.replica_idx}"
        owners = [r["lid"] for r in rep.get("routes", [])
                  if any(a.startswith("rs=") and a.endswith(suffix) for a in r.get("addresses") or [])]
        if len(owners) != 1:
            return None
        d = owners[0]
        return LogicalEndpointID(d["model_name"], int(d["stage_idx"]), int(d.get("shard_idx", 0)),
                                 int(d.get("replica_idx", 0)))

    return resolve

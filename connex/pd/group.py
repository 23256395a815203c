"""Transport peer-death events -> group failure reports (reference
``connex/pd/group.py``).

:class:`GroupFailureTracker` (pure logic) decides which peer LIDs to report:
a link must have been up before its failure counts, timeouts are only
suspicion (left to the lease), and each peer is reported once per
incarnation.  :class:`PeerDeathReporter` reads a transfer engine's events and
reports dead peers to the front router, which fails their whole group.
"""
from __future__ import annotations

import logging
import threading
import time
from typing import Callable, Iterable, List, Optional

from connex.protocol import LogicalEndpointID

log = logging.getLogger("connex.pd")


class GroupFailureTracker:
    def __init__(self, model: Optional[str], stages: Iterable[int]):
        self.model = model
        self.stages = {int(s) for s in stages}
        self.up: set = set()
        self.reported: set = set()

    def on_event(self, ev: dict) -> Optional[LogicalEndpointID]:
        peer = ev.get("peer")
        if not peer or len(peer) < 4:
            return None
        key = (peer[0], int(peer[1]), int(peer[2]), int(peer[3]))
        if key[1] not in self.stages or (self.model and key[0] != self.model):
            return None
        if ev.get("type") in ("up", "joined"):
            self.up.add(key)
            self.reported.discard(key)
            return None
        if ev.get("type") != "failed" or key not in self.up or key in self.reported:
            return None
        if "timeout" in str(ev.get("reason", "")):
            return None
        self.up.discard(key)
        self.reported.add(key)
        return LogicalEndpointID(*key)


class PeerDeathReporter:
    def __init__(self, engine, front_router_api: str, model: Optional[str], stages: Optional[Iterable[int]] = None,
                 report: Optional[Callable[[LogicalEndpointID, str], object]] = None,
                 resolve: Optional[Callable[[LogicalEndpointID], Optional[LogicalEndpointID]]] = None):
        if stages is None:
            from connex.pd.membership import PD_STAGE
            stages = PD_STAGE.values()
        self.engine = engine
        self.tracker = GroupFailureTracker(model, stages)
        self.front_router = front_router_api
        if report is None:
            from connex.pd.membership import report_failure

            def report(lid, reason):
                return report_failure(front_router_api, lid, reason)
        self._report = report
        self._resolve = resolve
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.reports: List[tuple] = []

    def start(self) -> None:
        self._thread = threading.Thread(target=self._run, name="connex-pd-peer-watch", daemon=True)
        self._thread.start()

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                ev = self.engine.wait_event(100)
            except Exception:
                return
            if ev is not None:
                self.handle(ev)

    def handle(self, ev: dict) -> Optional[LogicalEndpointID]:
        lid = self.tracker.on_event(ev)
        if lid is None:
            return None
        if self._resolve is not None:
            try:
                lid = self._resolve(lid)
            except Exception:
                lid = None
            if lid is None:
                return None
        reason = f"peer died ({ev.get('reason', 'transport event')})"
        log.warning("%s rank %d of replica %d died: reporting its group", lid.model_name, lid.shard_idx,
                    lid.replica_idx)
        try:
            res = self._report(lid, reason)
        except Exception as e:
            res = e
        self.reports.append((time.time(), lid, res))
        return lid

    def stop(self) -> None:
        self._stop.set()


def rs_port_resolver(front_router_api: str, model: str, timeout_ms: int = 1000):
    """Map transport identities that name a peer by its engine port
    (``(model, stage, 0, port)``) to the PD member advertising ``rs=host:port``."""
    from connex.pd.membership import PD_STAGE, _router_call

    def resolve(lid: LogicalEndpointID) -> Optional[LogicalEndpointID]:
        rep = _router_call(front_router_api, "get_routes",
                           {"model_name": model, "stage_idx": list(PD_STAGE.values()), "compact": True}, timeout_ms)
        if rep is None:
            return None
        port = str(lid.replica_idx)
        hits = []
        for r in rep.get("routes", []):
            if any(a.startswith("rs=") and a.rsplit(":", 1)[-1] == port for a in r.get("addresses") or []):
                d = r["lid"]
                hits.append(LogicalEndpointID(d["model_name"], int(d["stage_idx"]), int(d.get("shard_idx", 0)),
                                              int(d.get("replica_idx", 0))))
        return hits[0] if len(hits) == 1 else None

    return resolve

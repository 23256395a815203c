"""Front router: the production control plane (routes, epochs, leases, events).

Wire contract (the reference's ``connex/front_router.py``):

* JSON request/reply on a ZeroMQ REP socket (default ``tcp://*:15555``):
  ``{"method": m, "params": {...}}`` with methods ``register``, ``deregister``,
  ``heartbeat``, ``get_routes``, ``get_stage_routes``, ``get_route``,
  ``get_epoch``, ``prepare_migration``, ``scale_out``, ``shadow_ready``,
  ``execute_cutover``, ``get_stats``, ``get_topology``, ``update_route``,
  ``force_refresh``, ``report_failure`` (``front_router.py:1119-1136``).
* Events on a PUB socket (default ``tcp://*:15560``) as two frames:
  topic ``connex.<event_name>`` and the event JSON
  ``{"type", "epoch", "payload", "timestamp", "source_lid", "seq"}`` with a
  monotonic ``seq`` so clients can detect gaps (``:851-917``).

Semantics: routes indexed by stage with heartbeat-ordered expiry
(O(expired) per health check), ACTIVE -> UNHEALTHY after ``timeout`` without
heartbeat, removed (and announced as deregistered, reason ``expired``)
after a further ``grace``; an UNHEALTHY route that heartbeats again is
re-announced.  A *group* (``group_size`` > 1, e.g. the TP ranks of one
instance) is one endpoint: any shard failing, leaving or going unhealthy
fails every shard.  Migrations go prepare -> shadow_ready -> cutover ->
complete / abort with an epoch bump.
"""
from __future__ import annotations

import argparse
import json
import logging
import os
import threading
import time
from collections import OrderedDict
from dataclasses import asdict, dataclass, field
from enum import IntEnum
from typing import Any, Callable, Dict, List, Optional, Set, Tuple

import zmq

logger = logging.getLogger("connex.front_router")

ENV_HEARTBEAT_TIMEOUT = "CONNEX_HEARTBEAT_TIMEOUT_S"
ENV_HEALTH_CHECK_INTERVAL = "CONNEX_HEALTH_CHECK_INTERVAL_S"
ENV_UNHEALTHY_GRACE = "CONNEX_UNHEALTHY_GRACE_S"


def _env_float(name: str, default: float) -> float:
    raw = os.environ.get(name)
    if not raw:
        return default
    try:
        return float(raw)
    except ValueError:
        logger.warning("ignoring invalid %s=%r", name, raw)
        return default


class RouteState(IntEnum):
    UNKNOWN = 0
    ACTIVE = 1
    DRAINING = 2
    MIGRATING = 3
    UNHEALTHY = 4


class EventType(IntEnum):
    ENDPOINT_REGISTERED = 0
    ENDPOINT_DEREGISTERED = 1
    ENDPOINT_UNHEALTHY = 2
    EPOCH_BUMPED = 3
    PREPARE_MIGRATION = 4
    SHADOW_READY = 5
    CUTOVER_START = 6
    CUTOVER_COMPLETE = 7
    MIGRATION_FAILED = 8
    ROUTE_UPDATED = 9


class TransportCapability(IntEnum):
    ZEROMQ = 0
    UCX_TCP = 1
    UCX_RDMA = 2
    GPU_DIRECT = 3
    MOONCAKE_TE = 4
    NVLINK_P2P = 5


@dataclass
class LogicalEndpointID:
    model_name: str
    stage_idx: int
    shard_idx: int = 0
    replica_idx: int = 0

    def to_key(self) -> str:
        return f"{self.model_name}:{self.stage_idx}:{self.shard_idx}:{self.replica_idx}"

    @classmethod
    def from_key(cls, key: str) -> "LogicalEndpointID":
        p = key.split(":")
        return cls(p[0], int(p[1]), int(p[2]) if len(p) > 2 else 0, int(p[3]) if len(p) > 3 else 0)

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "LogicalEndpointID":
        return cls(d["model_name"], int(d["stage_idx"]), int(d.get("shard_idx", 0)), int(d.get("replica_idx", 0)))

    def __hash__(self):
        return hash(self.to_key())


def _caps(values) -> List[TransportCapability]:
    out = []
    for c in values or []:
        try:
            out.append(TransportCapability(int(c)))
        except ValueError:
            pass
    return out


@dataclass
class RouteEntry:
    lid: LogicalEndpointID
    addresses: List[str]
    capabilities: List[TransportCapability]
    epoch: int
    state: RouteState = RouteState.ACTIVE
    last_heartbeat: float = field(default_factory=time.time)
    registered_at: float = field(default_factory=time.time)
    metadata: Dict[str, Any] = field(default_factory=dict)

    @property
    def group_size(self) -> int:
        return int(self.metadata.get("group_size", 1) or 1)

    def to_dict(self) -> Dict[str, Any]:
        return {"lid": self.lid.to_dict(), "addresses": self.addresses,
                "capabilities": [int(c) for c in self.capabilities], "epoch": self.epoch,
                "state": int(self.state), "last_heartbeat": self.last_heartbeat,
                "registered_at": self.registered_at, "metadata": self.metadata}

    def to_compact_dict(self) -> Dict[str, Any]:
        d = {"lid": self.lid.to_dict(), "addresses": list(self.addresses),
             "capabilities": [int(c) for c in self.capabilities], "epoch": self.epoch,
             "state": int(self.state)}
        if self.group_size > 1:
            d["group_size"] = self.group_size
        return d

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "RouteEntry":
        md = dict(d.get("metadata") or {})
        if d.get("group_size"):
            md.setdefault("group_size", d["group_size"])
        return cls(lid=LogicalEndpointID.from_dict(d["lid"]), addresses=list(d["addresses"]),
                   capabilities=_caps(d.get("capabilities")), epoch=int(d.get("epoch", 0)),
                   state=RouteState(int(d.get("state", RouteState.ACTIVE))),
                   last_heartbeat=d.get("last_heartbeat", time.time()),
                   registered_at=d.get("registered_at", time.time()), metadata=md)


@dataclass
class Event:
    type: EventType
    epoch: int
    payload: Dict[str, Any]
    timestamp: float = field(default_factory=time.time)
    source_lid: Optional[str] = None
    seq: Optional[int] = None

    def to_dict(self) -> Dict[str, Any]:
        d = {"type": int(self.type), "epoch": self.epoch, "payload": self.payload,
             "timestamp": self.timestamp, "source_lid": self.source_lid}
        if self.seq is not None:
            d["seq"] = self.seq
        return d

    def serialize(self) -> bytes:
        return json.dumps(self.to_dict()).encode()

    @classmethod
    def deserialize(cls, data: bytes) -> "Event":
        d = json.loads(data.decode())
        return cls(EventType(d["type"]), d["epoch"], d["payload"], d.get("timestamp", time.time()),
                   d.get("source_lid"), d.get("seq"))

    @property
    def topic(self) -> str:
        return f"connex.{EventType(self.type).name.lower()}"


@dataclass
class MigrationRequest:
    migration_id: str
    lid: LogicalEndpointID
    old_address: str
    new_address: str
    old_epoch: int
    new_epoch: int
    state: str = "pending"  # pending, preparing, ready, cutting_over, complete, failed
    shadows_ready: Set[str] = field(default_factory=set)
    created_at: float = field(default_factory=time.time)
    completed_at: Optional[float] = None


# ------------------------------------------------------------- persistence
class PersistenceBackend:
    def get(self, key: str) -> Optional[Dict[str, Any]]:
        raise NotImplementedError

    def set(self, key: str, value: Dict[str, Any]) -> None:
        raise NotImplementedError

    def delete(self, key: str) -> None:
        raise NotImplementedError

    def get_all(self, prefix: str) -> Dict[str, Dict[str, Any]]:
        raise NotImplementedError


class InMemoryPersistence(PersistenceBackend):
    def __init__(self):
        self._d: Dict[str, Dict[str, Any]] = {}
        self._lock = threading.Lock()

    def get(self, key):
        with self._lock:
            return self._d.get(key)

    def set(self, key, value):
        with self._lock:
            self._d[key] = value

    def delete(self, key):
        with self._lock:
            self._d.pop(key, None)

    def get_all(self, prefix):
        with self._lock:
            return {k: v for k, v in self._d.items() if k.startswith(prefix)}


# ------------------------------------------------------------------- routes
class RouteManager:
    """Authoritative route table: by key, by (model, stage), and in heartbeat
    order (oldest first) so expiry walks only the expired prefix."""

    def __init__(self, persistence: Optional[PersistenceBackend] = None):
        self._routes: Dict[str, RouteEntry] = {}
        self._by_stage: Dict[Tuple[str, int], Dict[str, RouteEntry]] = {}
        self._hb: "OrderedDict[str, float]" = OrderedDict()
        self._lock = threading.RLock()
        self._p = persistence
        if self._p is not None:
            try:
                for r in sorted((RouteEntry.from_dict(v) for v in self._p.get_all("routes/").values()),
                                key=lambda r: r.last_heartbeat):
                    self._add(r.lid.to_key(), r)
            except Exception as e:
                logger.warning("route reload failed: %s", e)

    def _save(self, key: str, r: RouteEntry) -> None:
        if self._p is not None:
            self._p.set(f"routes/{key}", r.to_dict())

    def _add(self, key: str, r: RouteEntry) -> None:
        self._routes[key] = r
        self._by_stage.setdefault((r.lid.model_name, r.lid.stage_idx), {})[key] = r
        self._touch(key, r.last_heartbeat)

    def _pop(self, key: str) -> Optional[RouteEntry]:
        r = self._routes.pop(key, None)
        self._hb.pop(key, None)
        if r is not None:
            sk = (r.lid.model_name, r.lid.stage_idx)
            b = self._by_stage.get(sk)
            if b is not None:
                b.pop(key, None)
                if not b:
                    del self._by_stage[sk]
            if self._p is not None:
                self._p.delete(f"routes/{key}")
        return r

    def _touch(self, key: str, ts: float) -> None:
        self._hb[key] = ts
        self._hb.move_to_end(key)

    def add_route(self, lid, addresses, capabilities, epoch) -> RouteEntry:
        key = lid.to_key()
        now = time.time()
        with self._lock:
            r = self._routes.get(key)
            if r is not None:
                r.addresses, r.capabilities, r.epoch = list(addresses), list(capabilities), epoch
                r.state, r.last_heartbeat = RouteState.ACTIVE, now
                self._touch(key, now)
            else:
                r = RouteEntry(lid, list(addresses), list(capabilities), epoch, last_heartbeat=now)
                self._add(key, r)
            self._save(key, r)
            return r

    def get_route(self, lid) -> Optional[RouteEntry]:
        with self._lock:
            return self._routes.get(lid.to_key())

    def get_routes_for_model(self, model_name: str) -> List[RouteEntry]:
        with self._lock:
            return [r for r in self._routes.values() if r.lid.model_name == model_name]

    def get_routes_for_stage(self, model_name: str, stage_idx: int) -> List[RouteEntry]:
        with self._lock:
            b = self._by_stage.get((model_name, int(stage_idx)))
            rs = list(b.values()) if b else []
        return sorted(rs, key=lambda r: (r.lid.shard_idx, r.lid.replica_idx))

    def get_all_routes(self) -> List[RouteEntry]:
        with self._lock:
            return list(self._routes.values())

    def remove_route(self, lid) -> Optional[RouteEntry]:
        with self._lock:
            return self._pop(lid.to_key())

    def update_route_state(self, lid, state: RouteState) -> Optional[RouteEntry]:
        with self._lock:
            r = self._routes.get(lid.to_key())
            if r is not None:
                r.state = state
                self._save(lid.to_key(), r)
            return r

    def update_addresses(self, lid, addresses) -> Optional[Tuple[RouteEntry, List[str]]]:
        key = lid.to_key()
        with self._lock:
            r = self._routes.get(key)
            if r is None:
                return None
            old = list(r.addresses)
            r.addresses, r.last_heartbeat, r.state = list(addresses), time.time(), RouteState.ACTIVE
            self._touch(key, r.last_heartbeat)
            self._save(key, r)
            return r, old

    def apply_cutover(self, lid, addresses, epoch) -> Optional[RouteEntry]:
        with self._lock:
            r = self._routes.get(lid.to_key())
            if r is not None:
                r.addresses, r.epoch, r.state = list(addresses), epoch, RouteState.ACTIVE
                self._save(lid.to_key(), r)
            return r

    def heartbeat(self, lid) -> Tuple[bool, bool]:
        """(known, recovered-from-unhealthy)."""
        key = lid.to_key()
        with self._lock:
            r = self._routes.get(key)
            if r is None:
                return False, False
            r.last_heartbeat = time.time()
            self._touch(key, r.last_heartbeat)
            recovered = r.state == RouteState.UNHEALTHY
            if recovered:
                r.state = RouteState.ACTIVE
            return True, recovered

    def update_heartbeat(self, lid) -> bool:
        return self.heartbeat(lid)[0]

    def collect_expired(self, timeout_s: float, grace_s: float, now: Optional[float] = None):
        """ACTIVE older than timeout -> UNHEALTHY; UNHEALTHY older than
        timeout + grace -> removed.  Returns (newly_unhealthy, removed)."""
        now = time.time() if now is None else now
        cutoff, rm_cutoff = now - timeout_s, now - timeout_s - grace_s
        unhealthy, removed, dead_keys, retouch = [], [], [], []
        with self._lock:
            for key, ts in self._hb.items():
                if ts >= cutoff:
                    break
                r = self._routes.get(key)
                if r is None:
                    dead_keys.append(key)
                elif r.last_heartbeat >= cutoff:
                    retouch.append((key, r.last_heartbeat))
                elif r.state == RouteState.ACTIVE:
                    r.state = RouteState.UNHEALTHY
                    unhealthy.append(r)
                    self._save(key, r)
                elif r.state == RouteState.UNHEALTHY and r.last_heartbeat < rm_cutoff:
                    dead_keys.append(key)
            for key, ts in retouch:
                self._touch(key, ts)
            for key in dead_keys:
                r = self._pop(key)
                if r is not None:
                    removed.append(r)
        return unhealthy, removed

    def get_unhealthy_routes(self, timeout_s: float = 3.0) -> List[RouteEntry]:
        cutoff = time.time() - timeout_s
        with self._lock:
            out = []
            for key, ts in self._hb.items():
                if ts >= cutoff:
                    break
                r = self._routes.get(key)
                if r is not None and r.state == RouteState.ACTIVE:
                    out.append(r)
            return out


class EpochManager:
    def __init__(self, persistence: Optional[PersistenceBackend] = None):
        self._epoch = 0
        self._lock = threading.Lock()
        self._p = persistence
        self._history: List[Tuple[int, float, str]] = []
        if self._p is not None:
            d = self._p.get("epoch")
            if d:
                self._epoch = int(d.get("value", 0))

    @property
    def current(self) -> int:
        with self._lock:
            return self._epoch

    def bump(self, reason: str = "manual") -> int:
        with self._lock:
            self._epoch += 1
            self._history.append((self._epoch, time.time(), reason))
            del self._history[:-1000]
            if self._p is not None:
                self._p.set("epoch", {"value": self._epoch, "updated_at": time.time(), "reason": reason})
            return self._epoch

    def get_history(self, limit: int = 100):
        with self._lock:
            return self._history[-limit:]


class MemberManager:
    """Lease checker: timeout (default 3 s, env CONNEX_HEARTBEAT_TIMEOUT_S),
    grace (10 s, CONNEX_UNHEALTHY_GRACE_S), interval min(5, timeout/4)."""

    HEARTBEAT_TIMEOUT_S = 3.0
    GRACE_PERIOD_S = 10.0

    def __init__(self, route_manager: RouteManager, on_unhealthy: Optional[Callable] = None,
                 heartbeat_timeout_s: Optional[float] = None, grace_period_s: Optional[float] = None,
                 check_interval_s: Optional[float] = None, on_removed: Optional[Callable] = None):
        self._rm = route_manager
        self._on_unhealthy, self._on_removed = on_unhealthy, on_removed
        self.HEARTBEAT_TIMEOUT_S = heartbeat_timeout_s if heartbeat_timeout_s is not None else \
            _env_float(ENV_HEARTBEAT_TIMEOUT, type(self).HEARTBEAT_TIMEOUT_S)
        self.GRACE_PERIOD_S = grace_period_s if grace_period_s is not None else \
            _env_float(ENV_UNHEALTHY_GRACE, type(self).GRACE_PERIOD_S)
        dflt = min(5.0, max(0.05, self.HEARTBEAT_TIMEOUT_S / 4.0))
        self.check_interval_s = check_interval_s if check_interval_s is not None else \
            _env_float(ENV_HEALTH_CHECK_INTERVAL, dflt)
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    def start(self) -> None:
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, daemon=True, name="member-health-check")
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5.0)
            self._thread = None

    def _loop(self) -> None:
        while not self._stop.wait(self.check_interval_s):
            try:
                self._check_health()
            except Exception as e:  # keep checking
                logger.error("health check error: %s", e)

    def _check_health(self) -> None:
        unhealthy, removed = self._rm.collect_expired(self.HEARTBEAT_TIMEOUT_S, self.GRACE_PERIOD_S)
        for r in unhealthy:
            if self._on_unhealthy:
                try:
                    self._on_unhealthy(r.lid)
                except Exception as e:
                    logger.error("on_unhealthy failed: %s", e)
        for r in removed:
            if self._on_removed:
                try:
                    self._on_removed(r.lid)
                except Exception as e:
                    logger.error("on_removed failed: %s", e)


class EventBus:
    """PUB socket with a monotonic event ``seq`` and a bounded history."""

    def __init__(self, pub_address: str = "tcp://*:15560", max_history: int = 1000):
        self._addr = pub_address
        self._ctx: Optional[zmq.Context] = None
        self._pub: Optional[zmq.Socket] = None
        self._running = False
        self._lock = threading.Lock()
        self._history: List[Event] = []
        self._max_history = max_history
        self._seq = 0

    @property
    def seq(self) -> int:
        with self._lock:
            return self._seq

    def start(self) -> None:
        self._ctx = zmq.Context()
        self._pub = self._ctx.socket(zmq.PUB)
        self._pub.bind(self._addr)
        self._running = True

    def stop(self) -> None:
        self._running = False
        with self._lock:
            if self._pub is not None:
                self._pub.close(linger=0)
                self._pub = None
        if self._ctx is not None:
            self._ctx.term()
            self._ctx = None

    def publish(self, event: Event) -> None:
        with self._lock:
            if not self._running or self._pub is None:
                return
            self._seq += 1
            event.seq = self._seq
            self._history.append(event)
            del self._history[:-self._max_history]
            self._pub.send_multipart([event.topic.encode(), event.serialize()])

    def get_history(self, since_epoch: int = 0) -> List[Event]:
        with self._lock:
            return [e for e in self._history if e.epoch >= since_epoch]


class MigrationOrchestrator:
    """prepare (epoch bump, MIGRATING, PREPARE_MIGRATION) -> shadow_ready ->
    cutover (CUTOVER_START, route switched, CUTOVER_COMPLETE) or abort."""

    def __init__(self, route_manager: RouteManager, epoch_manager: EpochManager, event_bus: EventBus):
        self._rm, self._em, self._bus = route_manager, epoch_manager, event_bus
        self._pending: Dict[str, MigrationRequest] = {}
        self._lock = threading.Lock()

    def get(self, migration_id: str) -> Optional[MigrationRequest]:
        with self._lock:
            return self._pending.get(migration_id)

    def prepare_migration(self, lid: LogicalEndpointID, new_address: str) -> MigrationRequest:
        r = self._rm.get_route(lid)
        if r is None:
            raise ValueError(f"No route found for {lid.to_key()}")
        new_epoch = self._em.bump(f"migration:{lid.to_key()}")
        m = MigrationRequest(f"mig-{lid.to_key()}-{new_epoch}", lid, r.addresses[0] if r.addresses else "",
                             new_address, r.epoch, new_epoch)
        with self._lock:
            self._pending[m.migration_id] = m
        self._rm.update_route_state(lid, RouteState.MIGRATING)
        self._bus.publish(Event(EventType.PREPARE_MIGRATION, new_epoch,
                                {"migration_id": m.migration_id, "lid": lid.to_dict(),
                                 "old_address": m.old_address, "new_address": new_address,
                                 "old_epoch": r.epoch, "new_epoch": new_epoch}))
        return m

    def notify_shadow_ready(self, migration_id: str, from_lid: LogicalEndpointID) -> bool:
        with self._lock:
            m = self._pending.get(migration_id)
            if m is None:
                return False
            m.shadows_ready.add(from_lid.to_key())
            if m.state == "pending":
                m.state = "preparing"
        self._bus.publish(Event(EventType.SHADOW_READY, m.new_epoch,
                                {"migration_id": migration_id, "from_lid": from_lid.to_dict()}))
        return True

    def execute_cutover(self, migration_id: str) -> bool:
        with self._lock:
            m = self._pending.get(migration_id)
            if m is None or m.state not in ("pending", "preparing", "ready"):
                return False
            m.state = "cutting_over"
        self._bus.publish(Event(EventType.CUTOVER_START, m.new_epoch,
                                {"migration_id": migration_id, "lid": m.lid.to_dict()}))
        r = self._rm.apply_cutover(m.lid, [m.new_address], m.new_epoch)
        with self._lock:
            m.state, m.completed_at = "complete", time.time()
        payload = {"migration_id": migration_id, "lid": m.lid.to_dict(), "new_address": m.new_address}
        if r is not None:
            payload["route"] = r.to_compact_dict()
        self._bus.publish(Event(EventType.CUTOVER_COMPLETE, m.new_epoch, payload))
        return True

    def abort_migration(self, migration_id: str, reason: str) -> bool:
        with self._lock:
            m = self._pending.get(migration_id)
            if m is None or m.state in ("complete", "failed"):
                return False
            m.state = "failed"
        self._rm.update_route_state(m.lid, RouteState.ACTIVE)
        self._bus.publish(Event(EventType.MIGRATION_FAILED, m.new_epoch,
                                {"migration_id": migration_id, "lid": m.lid.to_dict(), "reason": reason}))
        return True


class FrontRouterConfig:
    def __init__(self, api_address: str = "tcp://*:15555", event_pub_address: str = "tcp://*:15560",
                 persistence_type: str = "memory", etcd_endpoints: Optional[List[str]] = None,
                 heartbeat_timeout_s: Optional[float] = None, grace_period_s: Optional[float] = None,
                 check_interval_s: Optional[float] = None):
        self.api_address = api_address
        self.event_pub_address = event_pub_address
        self.persistence_type = persistence_type
        self.etcd_endpoints = etcd_endpoints or ["localhost:2379"]
        self.heartbeat_timeout_s = heartbeat_timeout_s
        self.grace_period_s = grace_period_s
        self.check_interval_s = check_interval_s


class FrontRouter:
    def __init__(self, config: Optional[FrontRouterConfig] = None):
        self.config = config or FrontRouterConfig()
        if self.config.persistence_type != "memory":
            logger.warning("persistence %r is not available; using memory", self.config.persistence_type)
        self._persistence = InMemoryPersistence()
        self.route_manager = RouteManager(self._persistence)
        self.epoch_manager = EpochManager(self._persistence)
        self.event_bus = EventBus(self.config.event_pub_address)
        self.member_manager = MemberManager(self.route_manager, on_unhealthy=self._on_endpoint_unhealthy,
                                            heartbeat_timeout_s=self.config.heartbeat_timeout_s,
                                            grace_period_s=self.config.grace_period_s,
                                            check_interval_s=self.config.check_interval_s,
                                            on_removed=self._on_endpoint_expired)
        self.migration_orchestrator = MigrationOrchestrator(self.route_manager, self.epoch_manager,
                                                            self.event_bus)
        self._ctx: Optional[zmq.Context] = None
        self._api: Optional[zmq.Socket] = None
        self._running = False
        self._thread: Optional[threading.Thread] = None
        self._stats = {"registrations": 0, "deregistrations": 0, "heartbeats": 0, "migrations": 0,
                       "api_requests": 0}
        self._handlers = {
            "register": self._handle_register, "deregister": self._handle_deregister,
            "heartbeat": self._handle_heartbeat, "get_routes": self._handle_get_routes,
            "get_stage_routes": self._handle_get_stage_routes, "get_route": self._handle_get_route,
            "get_epoch": lambda p: {"epoch": self.epoch_manager.current},
            "prepare_migration": self._handle_prepare_migration, "scale_out": self._handle_scale_out,
            "shadow_ready": self._handle_shadow_ready, "execute_cutover": self._handle_execute_cutover,
            "get_stats": self._handle_get_stats, "get_topology": self._handle_get_topology,
            "update_route": self._handle_update_route, "force_refresh": self._handle_force_refresh,
            "report_failure": self._handle_report_failure,
        }

    # ---------------------------------------------------------- lifecycle
    def start(self) -> None:
        self.event_bus.start()
        self.member_manager.start()
        self._ctx = zmq.Context()
        self._api = self._ctx.socket(zmq.REP)
        self._api.bind(self.config.api_address)
        self._running = True
        self._thread = threading.Thread(target=self._api_loop, daemon=True, name="front-router-api")
        self._thread.start()

    def stop(self) -> None:
        self._running = False
        self.member_manager.stop()
        if self._thread is not None and self._thread is not threading.current_thread():
            self._thread.join(timeout=5.0)
        self._thread = None
        if self._api is not None:
            self._api.close(linger=0)
            self._api = None
        if self._ctx is not None:
            self._ctx.term()
            self._ctx = None
        self.event_bus.stop()

    def _api_loop(self) -> None:
        while self._running:
            try:
                if self._api.poll(timeout=200):
                    req = self._api.recv_json()
                    self._api.send_json(self._handle_request(req))
                    self._stats["api_requests"] += 1
            except Exception as e:
                if not self._running:
                    return
                logger.error("API error: %s", e)
                try:
                    self._api.send_json({"error": str(e)})
                except Exception:
                    pass

    def _handle_request(self, request: Dict[str, Any]) -> Dict[str, Any]:
        h = self._handlers.get(request.get("method", ""))
        if h is None:
            return {"error": f"Unknown method: {request.get('method', '')}"}
        try:
            return h(request.get("params", {}) or {})
        except Exception as e:
            logger.error("handler %s failed: %s", request.get("method"), e)
            return {"error": str(e)}

    # ------------------------------------------------------------ handlers
    def _handle_register(self, params):
        lid = LogicalEndpointID.from_dict(params["lid"])
        addresses = list(params["addresses"])
        caps = _caps(params.get("capabilities"))
        existing = self.route_manager.get_route(lid)
        is_reconnect = existing is not None
        old = list(existing.addresses) if existing else []
        changed = is_reconnect and set(old) != set(addresses)
        epoch = existing.epoch if existing else self.epoch_manager.current
        route = self.route_manager.add_route(lid, addresses, caps, epoch)
        g = int(params.get("group_size", 1) or 1)
        if g > 1:
            route.metadata["group_size"] = g
        else:
            route.metadata.pop("group_size", None)
        snapshot_seq = self.event_bus.seq  # read before the snapshot: events after it are replayable
        table = self.route_manager.get_routes_for_model(lid.model_name)
        self.event_bus.publish(Event(EventType.ENDPOINT_REGISTERED, epoch,
                                     {"lid": lid.to_dict(), "addresses": addresses, "is_reconnect": is_reconnect,
                                      "address_changed": changed, "old_addresses": old if changed else [],
                                      "route": route.to_compact_dict()}, source_lid=lid.to_key()))
        if changed:
            self._broadcast_route_updated(lid, old, addresses, epoch, route)
        self._stats["registrations"] += 1
        return {"success": True, "epoch": epoch, "is_reconnect": is_reconnect, "address_changed": changed,
                "route_table": [r.to_dict() for r in table], "seq": snapshot_seq}

    def _broadcast_route_updated(self, lid, old, new, epoch, route=None):
        route = route if route is not None else self.route_manager.get_route(lid)
        payload = {"lid": lid.to_dict(), "old_addresses": old, "new_addresses": new,
                   "stage_idx": lid.stage_idx, "replica_idx": lid.replica_idx}
        if route is not None:
            payload["route"] = route.to_compact_dict()
        self.event_bus.publish(Event(EventType.ROUTE_UPDATED, epoch, payload, source_lid=lid.to_key()))

    def _group_routes(self, lid) -> List[RouteEntry]:
        r = self.route_manager.get_route(lid)
        if r is None or r.group_size <= 1:
            return [r] if r is not None else []
        return [x for x in self.route_manager.get_routes_for_stage(lid.model_name, lid.stage_idx)
                if x.lid.replica_idx == lid.replica_idx and x.group_size > 1]

    def fail_group(self, lid, reason: str) -> List[str]:
        """Fail ``lid`` and, for a grouped endpoint, every shard of its group."""
        if not isinstance(lid, LogicalEndpointID):
            lid = LogicalEndpointID(lid.model_name, int(lid.stage_idx), int(lid.shard_idx), int(lid.replica_idx))
        failed = []
        for r in self._group_routes(lid):
            if self.route_manager.remove_route(r.lid) is None:
                continue
            failed.append(r.lid.to_key())
            self.event_bus.publish(Event(EventType.ENDPOINT_DEREGISTERED, self.epoch_manager.current,
                                         {"lid": r.lid.to_dict(), "reason": reason,
                                          "group": [lid.model_name, lid.stage_idx, lid.replica_idx],
                                          "cause": lid.to_key()}, source_lid=r.lid.to_key()))
        if failed:
            self._stats["group_failures"] = self._stats.get("group_failures", 0) + 1
        return failed

    def _handle_report_failure(self, params):
        failed = self.fail_group(LogicalEndpointID.from_dict(params["lid"]), str(params.get("reason") or "reported"))
        return {"success": bool(failed), "failed": failed}

    def _handle_deregister(self, params):
        lid = LogicalEndpointID.from_dict(params["lid"])
        existing = self.route_manager.get_route(lid)
        if existing is not None and existing.group_size > 1:
            failed = self.fail_group(lid, "group_left")
            self._stats["deregistrations"] += 1
            return {"success": bool(failed), "failed": failed}
        if self.route_manager.remove_route(lid) is None:
            return {"success": False, "error": "Route not found"}
        self.event_bus.publish(Event(EventType.ENDPOINT_DEREGISTERED, self.epoch_manager.current,
                                     {"lid": lid.to_dict()}, source_lid=lid.to_key()))
        self._stats["deregistrations"] += 1
        return {"success": True}

    def _handle_heartbeat(self, params):
        lid = LogicalEndpointID.from_dict(params["lid"])
        ok, recovered = self.route_manager.heartbeat(lid)
        self._stats["heartbeats"] += 1
        if recovered:
            r = self.route_manager.get_route(lid)
            if r is not None:
                self.event_bus.publish(Event(EventType.ENDPOINT_REGISTERED, self.epoch_manager.current,
                                             {"lid": lid.to_dict(), "addresses": list(r.addresses),
                                              "is_reconnect": True, "address_changed": False,
                                              "old_addresses": [], "recovered": True,
                                              "route": r.to_compact_dict()}, source_lid=lid.to_key()))
        return {"success": ok, "epoch": self.epoch_manager.current, "seq": self.event_bus.seq}

    def _handle_get_routes(self, params):
        seq = self.event_bus.seq  # before the snapshot
        model, stage = params.get("model_name"), params.get("stage_idx")
        if model and stage is not None:
            routes = []
            for st in (stage if isinstance(stage, list) else [stage]):
                routes.extend(self.route_manager.get_routes_for_stage(model, int(st)))
        elif model:
            routes = self.route_manager.get_routes_for_model(model)
        else:
            routes = self.route_manager.get_all_routes()
        out = [r.to_compact_dict() if params.get("compact") else r.to_dict() for r in routes]
        return {"routes": out, "epoch": self.epoch_manager.current, "seq": seq}

    def _handle_get_stage_routes(self, params):
        if params.get("model_name") is None or params.get("stage_idx") is None:
            return {"error": "model_name and stage_idx required"}
        q = dict(params)
        q.setdefault("compact", True)
        return self._handle_get_routes(q)

    def _handle_get_route(self, params):
        lid = LogicalEndpointID.from_dict(params["lid"])
        r = self.route_manager.get_route(lid)
        if r is not None and r.state == RouteState.ACTIVE:
            return {"route": r.to_dict()}
        if not params.get("allow_fallback", True):
            return {"route": r.to_dict()} if r is not None else {"error": "Route not found"}
        cands = [x for x in self.route_manager.get_routes_for_stage(lid.model_name, lid.stage_idx)
                 if x.lid.shard_idx == lid.shard_idx and x.lid.replica_idx != lid.replica_idx
                 and x.state == RouteState.ACTIVE]
        if cands:
            fb = cands[int(time.time() * 1000) % len(cands)]
            return {"route": fb.to_dict(), "is_fallback": True, "original_replica": lid.replica_idx,
                    "fallback_replica": fb.lid.replica_idx}
        if r is not None:
            return {"route": r.to_dict(), "warning": "Route not in ACTIVE state"}
        return {"error": f"Route not found for stage {lid.stage_idx} (no fallback available)"}

    def _handle_prepare_migration(self, params):
        try:
            m = self.migration_orchestrator.prepare_migration(LogicalEndpointID.from_dict(params["lid"]),
                                                              params["new_address"])
        except Exception as e:
            return {"success": False, "error": str(e)}
        self._stats["migrations"] += 1
        return {"success": True, "migration_id": m.migration_id, "new_epoch": m.new_epoch}

    def _handle_scale_out(self, params):
        if params.get("model_name") is None or params.get("stage_idx") is None or params.get("new_address") is None:
            return {"success": False, "error": "model_name, stage_idx, new_address required"}
        lid = LogicalEndpointID(params["model_name"], int(params["stage_idx"]), int(params.get("shard_idx", 0)),
                                int(params.get("replica_idx", 0)))
        try:
            m = self.migration_orchestrator.prepare_migration(lid, params["new_address"])
        except Exception as e:
            return {"success": False, "error": str(e)}
        self._stats["migrations"] += 1
        return {"success": True, "migration_id": m.migration_id, "new_epoch": m.new_epoch, "lid": lid.to_dict()}

    def _handle_get_topology(self, params):
        m = params.get("model_name")
        rs = self.route_manager.get_routes_for_model(m) if m else self.route_manager.get_all_routes()
        return {"routes": [r.to_dict() for r in rs], "epoch": self.epoch_manager.current}

    def _handle_shadow_ready(self, params):
        return {"success": self.migration_orchestrator.notify_shadow_ready(
            params["migration_id"], LogicalEndpointID.from_dict(params["from_lid"]))}

    def _handle_execute_cutover(self, params):
        return {"success": self.migration_orchestrator.execute_cutover(params["migration_id"])}

    def get_stats(self) -> Dict[str, Any]:
        return {"stats": dict(self._stats), "routes_count": len(self.route_manager.get_all_routes()),
                "current_epoch": self.epoch_manager.current}

    def _handle_get_stats(self, params):
        return self.get_stats()

    def _handle_update_route(self, params):
        lid = LogicalEndpointID.from_dict(params["lid"])
        res = self.route_manager.update_addresses(lid, list(params["addresses"]))
        if res is None:
            return {"success": False, "error": "Route not found"}
        r, old = res
        self._broadcast_route_updated(lid, old, list(params["addresses"]), r.epoch, r)
        return {"success": True, "old_addresses": old, "new_addresses": list(params["addresses"])}

    def _handle_force_refresh(self, params):
        m = params.get("model_name")
        rs = self.route_manager.get_routes_for_model(m) if m else self.route_manager.get_all_routes()
        n = 0
        for r in rs:
            if r.state == RouteState.ACTIVE:
                self._broadcast_route_updated(r.lid, r.addresses, r.addresses, r.epoch, r)
                n += 1
        return {"success": True, "refreshed_count": n}

    # ------------------------------------------------------- lease events
    def _on_endpoint_unhealthy(self, lid) -> None:
        r = self.route_manager.get_route(lid)
        if r is not None and r.group_size > 1:
            self.fail_group(lid, "group_member_unhealthy")
            return
        self.event_bus.publish(Event(EventType.ENDPOINT_UNHEALTHY, self.epoch_manager.current,
                                     {"lid": lid.to_dict()}))

    def _on_endpoint_expired(self, lid) -> None:
        self.event_bus.publish(Event(EventType.ENDPOINT_DEREGISTERED, self.epoch_manager.current,
                                     {"lid": lid.to_dict(), "reason": "expired"}, source_lid=lid.to_key()))


def main() -> None:
    p = argparse.ArgumentParser(description="connex front router")
    p.add_argument("--api-address", default="tcp://*:15555")
    p.add_argument("--event-address", default="tcp://*:15560")
    p.add_argument("--persistence", default="memory", choices=["memory", "etcd", "redis"])
    p.add_argument("--log-level", default="INFO", choices=["DEBUG", "INFO", "WARNING", "ERROR"])
    a = p.parse_args()
    logging.basicConfig(level=getattr(logging, a.log_level),
                        format="%(asctime)s [%(levelname)s] %(name)s: %(message)s")
    router = FrontRouter(FrontRouterConfig(a.api_address, a.event_address, a.persistence))
    router.start()
    try:
        while True:
            time.sleep(1)
    except KeyboardInterrupt:
        pass
    finally:
        router.stop()


if __name__ == "__main__":
    main()

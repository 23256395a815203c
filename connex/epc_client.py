"""EPC v2 client: an engine's connection to the front router.

* **Registration** of this engine's LID (with ``group_size`` for TP groups)
  and deregistration on stop.
* **Liveness**: a fixed-rate heartbeat on its *own* self-healing request
  channel, so a slow route query never delays it; a rejected heartbeat
  (the router forgot us) re-registers.
* **Routes**: :class:`RouteTableCache` is an event-sourced copy of the
  router's route table for this model.  Every router event carries a global
  ``seq``; the cache applies events in seq order and knows when it is in
  sync.  A gap in the seqs -- or a heartbeat showing the router ahead of the
  last applied event for a whole heartbeat -- marks the cache stale and one
  full snapshot re-syncs it.  Stage-scoped queries replace one stage's
  routes without a full refresh.
* **Migrations**: prepared shadow connections to a migration target, the
  ``shadow_ready`` answer, cut-over and abort bookkeeping.
* Address updates and failure reports.

``serving_routes`` is the group rule: an ungrouped route serves; a group
(``group_size`` > 1) serves through its shard 0, and only while all of its
shards are registered.

Wire parity: the JSON methods and event fields of
``connex/epc_client.py:142-1303`` / ``connex/front_router.py`` in the
reference; the decomposition here is this module's own.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import zmq

from connex.front_router import (Event as _RouterEvent, EventType, LogicalEndpointID, RouteState,
                                 TransportCapability)

logger = logging.getLogger("connex.epc_client")

ENV_HEARTBEAT_INTERVAL = "CONNEX_HEARTBEAT_INTERVAL_S"
ENV_API_TIMEOUT_MS = "CONNEX_EPC_API_TIMEOUT_MS"
ENV_HEARTBEAT_TIMEOUT_MS = "CONNEX_EPC_HEARTBEAT_TIMEOUT_MS"


def _env_float(name: str, default: float) -> float:
    try:
        return float(os.environ.get(name) or default)
    except ValueError:
        return default


@dataclass
class RouteEntry:
    """Client view of a route."""

    lid: LogicalEndpointID
    addresses: List[str]
    capabilities: List[TransportCapability]
    epoch: int
    state: RouteState = RouteState.ACTIVE
    group_size: int = 1

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "RouteEntry":
        caps = []
        for c in d.get("capabilities") or []:
            try:
                caps.append(TransportCapability(int(c)))
            except ValueError:
                continue                        # a capability this client does not know
        group = d.get("group_size") or (d.get("metadata") or {}).get("group_size") or 1
        return cls(lid=LogicalEndpointID.from_dict(d["lid"]), addresses=list(d.get("addresses") or []),
                   capabilities=caps, epoch=int(d.get("epoch", 0)),
                   state=RouteState(int(d.get("state", RouteState.ACTIVE))), group_size=int(group))


def serving_routes(routes: List[RouteEntry]) -> List[RouteEntry]:
    """Routes that serve traffic: ungrouped ones, and shard 0 of complete groups."""
    shards: Dict[tuple, set] = {}
    for r in routes:
        if r.group_size > 1:
            shards.setdefault((r.lid.model_name, r.lid.stage_idx, r.lid.replica_idx), set()).add(r.lid.shard_idx)

    def serves(r: RouteEntry) -> bool:
        if r.group_size <= 1:
            return True
        present = shards[(r.lid.model_name, r.lid.stage_idx, r.lid.replica_idx)]
        return r.lid.shard_idx == 0 and present >= set(range(r.group_size))
    return [r for r in routes if serves(r)]


@dataclass
class Event(_RouterEvent):
    """A router event plus whether the local route cache absorbed it."""

    cache_synced: bool = False

    @classmethod
    def deserialize(cls, data: bytes) -> "Event":
        e = _RouterEvent.deserialize(data)
        return cls(e.type, e.epoch, e.payload, e.timestamp, e.source_lid, e.seq)


@dataclass
class EPCV2ClientConfig:
    front_router_api: str = "tcp://localhost:15555"
    front_router_events: str = "tcp://localhost:15560"
    model_name: str = "default"
    stage_idx: int = 0
    shard_idx: int = 0
    replica_idx: int = 0
    group_size: int = 1
    local_addresses: List[str] = field(default_factory=list)
    capabilities: List[TransportCapability] = field(default_factory=list)
    heartbeat_interval_s: float = field(default_factory=lambda: _env_float(ENV_HEARTBEAT_INTERVAL, 1.0))
    api_timeout_ms: int = field(default_factory=lambda: int(_env_float(ENV_API_TIMEOUT_MS, 5000)))
    heartbeat_timeout_ms: Optional[int] = field(
        default_factory=lambda: int(_env_float(ENV_HEARTBEAT_TIMEOUT_MS, 0)) or None)
    ucx_enabled: bool = True
    gpu_direct_enabled: bool = False
    mooncake_enabled: bool = False

    @property
    def lid(self) -> LogicalEndpointID:
        return LogicalEndpointID(self.model_name, self.stage_idx, self.shard_idx, self.replica_idx)


# outcomes of RouteTableCache.apply
APPLIED, DUPLICATE, GAP, UNUSABLE = "applied", "duplicate", "gap", "unusable"


class RouteTableCache:
    """Event-sourced local copy of the router's routes for one model.

    ``seq`` is the last router event reflected here (None before the first
    snapshot); ``stale`` means events may be missing and a snapshot must
    come next.  Snapshots older than ``seq`` are ignored unless stale."""

    def __init__(self, model_name: Optional[str] = None):
        self.model = model_name
        self._routes: Dict[str, RouteEntry] = {}
        self._epoch = 0
        self._seq: Optional[int] = None
        self.stale = False
        self._router_seq_seen: Optional[int] = None
        self._lock = threading.RLock()
        self._callbacks: List[Callable[[RouteEntry], None]] = []

    # ----------------------------------------------------------- sync state
    @property
    def lock(self) -> threading.RLock:
        return self._lock

    @property
    def seq(self) -> Optional[int]:
        return self._seq

    @seq.setter
    def seq(self, value: Optional[int]) -> None:
        with self._lock:
            self._seq = value

    @property
    def epoch(self) -> int:
        return self._epoch

    @property
    def in_sync(self) -> bool:
        with self._lock:
            return self._seq is not None and not self.stale

    def _older(self, seq: Optional[int]) -> bool:
        return seq is not None and self._seq is not None and seq < self._seq and not self.stale

    def note_router_seq(self, router_seq: Optional[int]) -> None:
        """The router's seq as a heartbeat reported it.  If the seq reported
        one heartbeat ago is still ahead of the last applied event, events
        were lost: mark the cache stale."""
        if router_seq is None:
            return
        with self._lock:
            prev, self._router_seq_seen = self._router_seq_seen, router_seq
            if prev is not None and (self._seq is None or self._seq < prev):
                self.stale = True

    # ------------------------------------------------------------- updates
    def load(self, routes: List[Dict[str, Any]], epoch: int, seq: Optional[int] = None) -> bool:
        """A full snapshot taken at ``seq``; False when it is older than the cache."""
        with self._lock:
            if self._older(seq):
                return False
            self._routes = {}
            for d in routes:
                r = RouteEntry.from_dict(d)
                self._routes[r.lid.to_key()] = r
            self._epoch = epoch
            if seq is not None:
                self._seq, self.stale = seq, False
            return True

    def update_from_list(self, routes: List[Dict[str, Any]], epoch: int) -> None:
        self.load(routes, epoch)

    def replace_stage(self, model_name: str, stage_idx: int, routes: List[RouteEntry], epoch: int,
                      seq: Optional[int] = None) -> bool:
        """One stage's routes from a stage query taken at ``seq``."""
        with self._lock:
            if self._older(seq):
                return False
            self._routes = {k: r for k, r in self._routes.items()
                            if not (r.lid.model_name == model_name and r.lid.stage_idx == stage_idx)}
            for r in routes:
                self._routes[r.lid.to_key()] = r
            self._epoch = max(self._epoch, epoch)
            return True

    def _mutate(self, event: Event) -> bool:
        """Reflect one event in the routes; False if it cannot be applied
        (an update without its route)."""
        p = event.payload or {}
        if p.get("lid") is None:
            return True
        lid = LogicalEndpointID.from_dict(p["lid"])
        if self.model is not None and lid.model_name != self.model:
            return True
        kind = event.type
        if kind in (EventType.ENDPOINT_REGISTERED, EventType.ROUTE_UPDATED, EventType.CUTOVER_COMPLETE):
            if "route" not in p:
                return False
            self.upsert(RouteEntry.from_dict(p["route"]), event.epoch)
        elif kind == EventType.ENDPOINT_DEREGISTERED:
            self.remove(lid)
        elif kind in (EventType.ENDPOINT_UNHEALTHY, EventType.PREPARE_MIGRATION, EventType.MIGRATION_FAILED):
            state = {EventType.ENDPOINT_UNHEALTHY: RouteState.UNHEALTHY,
                     EventType.PREPARE_MIGRATION: RouteState.MIGRATING,
                     EventType.MIGRATION_FAILED: RouteState.ACTIVE}[kind]
            self.set_state(lid, state)
        return True

    def apply(self, event: Event) -> str:
        """Apply the next event: APPLIED, DUPLICATE (already reflected), GAP
        (events are missing: stale now) or UNUSABLE (stale now)."""
        with self._lock:
            if self._seq is not None and event.seq <= self._seq and not self.stale:
                return DUPLICATE
            if self._seq is None or self.stale or event.seq != self._seq + 1:
                self.stale = True
                return GAP
            if not self._mutate(event):
                self.stale = True
                return UNUSABLE
            self._seq = event.seq
            return APPLIED

    # -------------------------------------------------------- single routes
    def upsert(self, route: RouteEntry, epoch: int = 0) -> None:
        with self._lock:
            self._routes[route.lid.to_key()] = route
            self._epoch = max(self._epoch, epoch)

    def update_single(self, route: RouteEntry, epoch: int) -> None:
        self.upsert(route, epoch)
        for cb in list(self._callbacks):
            try:
                cb(route)
            except Exception as e:  # noqa: BLE001
                logger.error("route callback failed: %s", e)

    def remove(self, lid: LogicalEndpointID) -> None:
        with self._lock:
            self._routes.pop(lid.to_key(), None)

    def set_state(self, lid: LogicalEndpointID, state: RouteState) -> bool:
        with self._lock:
            r = self._routes.get(lid.to_key())
            if r is not None:
                r.state = state
            return r is not None

    def add_callback(self, callback: Callable[[RouteEntry], None]) -> None:
        self._callbacks.append(callback)

    # ---------------------------------------------------------------- reads
    def get(self, lid: LogicalEndpointID) -> Optional[RouteEntry]:
        with self._lock:
            return self._routes.get(lid.to_key())

    def get_all(self) -> List[RouteEntry]:
        with self._lock:
            return list(self._routes.values())

    def get_for_model(self, model_name: str) -> List[RouteEntry]:
        with self._lock:
            return serving_routes([r for r in self._routes.values() if r.lid.model_name == model_name])

    def get_for_stage(self, model_name: str, stage_idx: int) -> List[RouteEntry]:
        with self._lock:
            mine = [r for r in self._routes.values() if r.lid.model_name == model_name and r.lid.stage_idx == stage_idx]
        return sorted(serving_routes(mine), key=lambda r: (r.lid.shard_idx, r.lid.replica_idx))


class DataPlaneManager:
    """Bookkeeping of per-(LID, address) data-plane connections."""

    def __init__(self, config: EPCV2ClientConfig):
        self._config = config
        self._conns: Dict[str, Dict[str, Any]] = {}
        self._lock = threading.Lock()

    def get_or_create_connection(self, lid: LogicalEndpointID, address: str) -> Dict[str, Any]:
        with self._lock:
            return self._conns.setdefault(f"{lid.to_key()}@{address}",
                                          {"lid": lid, "address": address, "created_at": time.time()})

    def close_connection(self, lid: LogicalEndpointID) -> None:
        prefix = lid.to_key() + "@"
        with self._lock:
            self._conns = {k: v for k, v in self._conns.items() if not k.startswith(prefix)}

    def close_all(self) -> None:
        with self._lock:
            self._conns.clear()

    def connections(self) -> List[str]:
        with self._lock:
            return list(self._conns)


class ShadowConnectionManager:
    """Connections to a migration target built before the cut-over."""

    def __init__(self, data_plane: DataPlaneManager):
        self._dp = data_plane
        self._shadows: Dict[str, Dict[str, Any]] = {}
        self._lock = threading.Lock()

    def prepare_shadow(self, migration_id: str, lid: LogicalEndpointID, new_address: str) -> bool:
        with self._lock:
            self._shadows.setdefault(migration_id, {
                "lid": lid, "new_address": new_address, "ready": True, "created_at": time.time(),
                "connection": self._dp.get_or_create_connection(lid, new_address)})
            return True

    def activate_shadow(self, migration_id: str) -> bool:
        with self._lock:
            return self._shadows.pop(migration_id, None) is not None

    def discard_shadow(self, migration_id: str) -> None:
        with self._lock:
            self._shadows.pop(migration_id, None)

    def pending(self) -> List[str]:
        with self._lock:
            return list(self._shadows)


class APITimeoutError(RuntimeError):
    """A front-router request got no reply in time."""


class _Requester:
    """Serialised request/reply on a REQ socket.  A REQ socket that missed
    its reply is stuck in the wrong state, so after any timeout or ZMQ error
    the socket is thrown away and the next call opens a fresh one."""

    def __init__(self, context: zmq.Context, endpoint: str, timeout_ms: int, name: str):
        self._ctx, self._endpoint, self.timeout_ms, self._name = context, endpoint, int(timeout_ms), name
        self._lock = threading.Lock()
        self._sock: Optional[zmq.Socket] = None
        self._closed = False
        self.resets = 0

    def _socket(self) -> zmq.Socket:
        if self._sock is None:
            s = self._ctx.socket(zmq.REQ)
            for opt, val in ((zmq.LINGER, 0), (zmq.SNDTIMEO, self.timeout_ms), (zmq.RCVTIMEO, self.timeout_ms)):
                s.setsockopt(opt, val)
            s.connect(self._endpoint)
            self._sock = s
        return self._sock

    def _discard(self) -> None:
        if self._sock is not None:
            try:
                self._sock.close(linger=0)
            except Exception:  # noqa: BLE001
                pass
            self._sock = None
            self.resets += 1

    def call(self, request: Dict[str, Any], timeout_ms: Optional[int] = None) -> Dict[str, Any]:
        wait = self.timeout_ms if timeout_ms is None else int(timeout_ms)
        with self._lock:
            if self._closed:
                raise RuntimeError("Not connected to Front Router")
            s = self._socket()
            try:
                s.send_json(request)
                if s.poll(wait, zmq.POLLIN):
                    return s.recv_json()
            except zmq.ZMQError as e:
                self._discard()
                raise RuntimeError(f"{self._name}: ZMQ error: {e}") from e
            self._discard()
            raise APITimeoutError(f"{self._name}: no reply to {request.get('method')!r} within {wait} ms")

    def close(self) -> None:
        with self._lock:
            self._closed = True
            self._discard()


_ReqChannel = _Requester        # earlier name


class EPCV2Client:
    def __init__(self, config: EPCV2ClientConfig):
        self.config = config
        self.lid = config.lid
        self._ctx: Optional[zmq.Context] = None
        self._api: Optional[_Requester] = None
        self._hb: Optional[_Requester] = None
        self._sub: Optional[zmq.Socket] = None
        self.route_table = RouteTableCache(config.model_name)
        self._data_plane = DataPlaneManager(config)
        self._shadow_manager = ShadowConnectionManager(self._data_plane)
        self._registered = False
        self._running = False
        self._local_epoch = 0
        self._stop_event = threading.Event()
        self._stage_query_supported = True
        self.stats: Dict[str, int] = {"full_refreshes": 0, "stage_queries": 0, "incremental_applied": 0,
                                      "seq_gaps": 0, "heartbeat_failures": 0}
        self._heartbeat_thread: Optional[threading.Thread] = None
        self._event_thread: Optional[threading.Thread] = None
        self._event_handlers: Dict[EventType, List[Callable[[Event], None]]] = {}
        self._pending_migrations: Dict[str, Dict[str, Any]] = {}
        self._builtin = {EventType.ENDPOINT_REGISTERED: self._on_endpoint_registered,
                         EventType.ENDPOINT_DEREGISTERED: self._on_endpoint_deregistered,
                         EventType.PREPARE_MIGRATION: self._on_prepare_migration,
                         EventType.CUTOVER_START: self._on_cutover_start,
                         EventType.CUTOVER_COMPLETE: self._on_cutover_complete,
                         EventType.MIGRATION_FAILED: self._on_migration_failed,
                         EventType.ROUTE_UPDATED: self._on_route_updated}

    # ------------------------------------------------------------ lifecycle
    def _heartbeat_timeout_ms(self) -> int:
        if self.config.heartbeat_timeout_ms:
            return int(self.config.heartbeat_timeout_ms)
        return int(min(self.config.api_timeout_ms, max(500, self.config.heartbeat_interval_s * 1000)))

    def _open(self) -> None:
        self._ctx = zmq.Context()
        self._stop_event.clear()
        self._api = _Requester(self._ctx, self.config.front_router_api, self.config.api_timeout_ms, "epc-api")
        self._hb = _Requester(self._ctx, self.config.front_router_api, self._heartbeat_timeout_ms(), "epc-heartbeat")
        self._sub = self._ctx.socket(zmq.SUB)
        self._sub.setsockopt(zmq.LINGER, 0)
        self._sub.connect(self.config.front_router_events)
        self._sub.setsockopt_string(zmq.SUBSCRIBE, "connex.")

    def _spawn(self, target, name: str) -> threading.Thread:
        t = threading.Thread(target=target, daemon=True, name=f"{name}-{self.lid.stage_idx}")
        t.start()
        return t

    def start(self) -> bool:
        try:
            self._open()
            self._running = True
            if not self._register():
                self.stop()
                return False
            self._event_thread = self._spawn(self._event_loop, "epc-events")
            self._heartbeat_thread = self._spawn(self._heartbeat_loop, "epc-heartbeat")
            return True
        except Exception as e:  # noqa: BLE001
            logger.error("EPC client start failed: %s", e)
            self.stop()
            return False

    def stop(self, deregister: bool = True) -> None:
        self._running = False
        self._stop_event.set()
        me = threading.current_thread()
        for t in (self._heartbeat_thread, self._event_thread):
            if t is not None and t is not me and t.is_alive():
                t.join(timeout=2.0)
        self._heartbeat_thread = self._event_thread = None
        if deregister and self._registered and self._api is not None:
            self._deregister()
        if self._sub is not None:
            self._sub.close(linger=0)
            self._sub = None
        for ch in (self._api, self._hb):
            if ch is not None:
                ch.close()
        self._api = self._hb = None
        if self._ctx is not None:
            self._ctx.term()
            self._ctx = None
        self._data_plane.close_all()
        self._registered = False

    def kill(self) -> None:
        """Stop without deregistering (as if the process died): the router
        learns only through the missed lease.  Used by failure tests."""
        self.stop(deregister=False)

    # ------------------------------------------------------------------ api
    def call(self, method: str, params: Dict[str, Any], channel: Optional[_Requester] = None,
             timeout_ms: Optional[int] = None) -> Dict[str, Any]:
        """One front-router JSON request; raises on an ``error`` reply."""
        ch = channel if channel is not None else self._api
        if ch is None:
            raise RuntimeError("Not connected to Front Router")
        resp = ch.call({"method": method, "params": params}, timeout_ms)
        if "error" in resp:
            raise RuntimeError(f"API error: {resp['error']}")
        return resp

    _call_api = call

    def _register(self, channel: Optional[_Requester] = None) -> bool:
        params = {"lid": self.lid.to_dict(), "addresses": list(self.config.local_addresses),
                  "capabilities": [int(c) for c in self.config.capabilities]}
        if self.config.group_size > 1:
            params["group_size"] = int(self.config.group_size)
        try:
            resp = self.call("register", params, channel=channel)
        except Exception as e:  # noqa: BLE001
            logger.error("registration failed: %s", e)
            return False
        if not resp.get("success"):
            return False
        self._local_epoch = resp.get("epoch", 0)
        self._registered = True
        self.route_table.load(resp.get("route_table", []), self._local_epoch, resp.get("seq"))
        return True

    def _deregister(self) -> None:
        try:
            self.call("deregister", {"lid": self.lid.to_dict()})
            self._registered = False
        except Exception as e:  # noqa: BLE001
            logger.warning("deregistration failed: %s", e)

    def _send_heartbeat(self) -> bool:
        try:
            resp = self.call("heartbeat", {"lid": self.lid.to_dict()}, channel=self._hb)
        except Exception as e:  # noqa: BLE001
            self.stats["heartbeat_failures"] += 1
            logger.debug("heartbeat failed: %s", e)
            return False
        self._local_epoch = max(self._local_epoch, resp.get("epoch", 0))
        self.route_table.note_router_seq(resp.get("seq"))
        if resp.get("success"):
            return True
        if self._running:
            logger.warning("heartbeat rejected (unknown endpoint): re-registering")
            return self._register(channel=self._hb)
        return False

    def _heartbeat_loop(self) -> None:
        period = max(0.01, float(self.config.heartbeat_interval_s))
        due = time.monotonic()
        while self._running:
            if self._registered:
                self._send_heartbeat()
            due = max(due + period, time.monotonic())      # fixed rate; no burst after a stall
            if self._stop_event.wait(due - time.monotonic()):
                break

    # --------------------------------------------------------------- routes
    def refresh_routes(self) -> List[RouteEntry]:
        """Load a full snapshot of this model's routes."""
        try:
            resp = self.call("get_routes", {"model_name": self.lid.model_name})
        except Exception as e:  # noqa: BLE001
            logger.error("route refresh failed: %s", e)
            return []
        epoch = resp.get("epoch", self._local_epoch)
        self.route_table.load(resp.get("routes", []), epoch, resp.get("seq"))
        self._local_epoch = max(self._local_epoch, epoch)
        self.stats["full_refreshes"] += 1
        return self.route_table.get_all()

    def cache_in_sync(self) -> bool:
        return self.route_table.in_sync and self._event_thread is not None and self._event_thread.is_alive()

    def _stage_query(self, stage_idx: int) -> Optional[dict]:
        if not self._stage_query_supported:
            return None
        try:
            return self.call("get_stage_routes", {"model_name": self.lid.model_name, "stage_idx": int(stage_idx)})
        except RuntimeError as e:
            if "Unknown method" not in str(e):
                raise
            self._stage_query_supported = False    # an older router: full refreshes instead
            return None

    def query_stage_routes(self, stage_idx: int) -> Optional[List[RouteEntry]]:
        """One stage's serving routes straight from the router (None on failure)."""
        model = self.lid.model_name
        try:
            resp = self._stage_query(stage_idx)
            if resp is None:
                self.refresh_routes()
                return self.route_table.get_for_stage(model, int(stage_idx))
            self.stats["stage_queries"] += 1
            entries = [RouteEntry.from_dict(r) for r in resp.get("routes", [])]
            self.route_table.replace_stage(model, int(stage_idx), entries, resp.get("epoch", self._local_epoch),
                                           resp.get("seq"))
            return sorted(serving_routes(entries), key=lambda r: (r.lid.shard_idx, r.lid.replica_idx))
        except Exception as e:  # noqa: BLE001
            logger.warning("stage %s route query failed: %s", stage_idx, e)
            return None

    def get_stage_peers(self, stage_idx: int, refresh: str = "auto") -> List[RouteEntry]:
        """Routes of a stage: ``never`` = cache only; ``auto`` = cache while it
        is event-synced, else a stage query; ``always`` = a stage query."""
        if refresh not in ("never", "auto", "always"):
            raise ValueError(f"invalid refresh mode: {refresh!r}")
        if refresh == "always" or (refresh == "auto" and not self.cache_in_sync()):
            fresh = self.query_stage_routes(stage_idx)
            if fresh is not None:
                return fresh
        return self.route_table.get_for_stage(self.lid.model_name, int(stage_idx))

    # --------------------------------------------------------------- events
    def _event_loop(self) -> None:
        last_resync = 0.0
        while self._running:
            try:
                if self._sub.poll(timeout=200):
                    _topic, data = self._sub.recv_multipart()
                    self._handle_event(Event.deserialize(data))
                elif self.route_table.stale and self._running and time.monotonic() - last_resync > 1.0:
                    last_resync = time.monotonic()        # stale without new events: re-sync by snapshot
                    self.refresh_routes()
            except Exception as e:  # noqa: BLE001
                if self._running:
                    logger.error("event loop error: %s", e)

    def _absorb(self, event: Event) -> bool:
        """Reflect ``event`` in the route cache; True when the cache is in
        sync with it afterwards (re-synced by a snapshot on a gap)."""
        if event.seq is None:
            return False
        outcome = self.route_table.apply(event)
        if outcome == APPLIED:
            self.stats["incremental_applied"] += 1
            return True
        if outcome == DUPLICATE:
            return True
        if outcome == GAP:
            self.stats["seq_gaps"] += 1
            self.refresh_routes()
            if not self.route_table.in_sync:
                return False
            if event.seq <= self.route_table.seq:
                return True                        # the snapshot already includes it
            again = self.route_table.apply(event)
            if again == APPLIED:
                self.stats["incremental_applied"] += 1
            return again in (APPLIED, DUPLICATE)
        return False

    def _handle_event(self, event: Event) -> None:
        self._local_epoch = max(self._local_epoch, event.epoch)
        try:
            event.cache_synced = self._absorb(event)
        except Exception as e:  # noqa: BLE001
            logger.error("route cache sync error: %s", e)
            event.cache_synced = False
        if event.source_lid == self.lid.to_key():
            return                                 # our own registration / update
        handlers = [self._builtin[event.type]] if event.type in self._builtin else []
        for h in handlers + list(self._event_handlers.get(event.type, [])):
            try:
                h(event)
            except Exception as e:  # noqa: BLE001
                logger.error("event handler error: %s", e)

    def _event_lid(self, event: Event) -> LogicalEndpointID:
        return LogicalEndpointID.from_dict(event.payload["lid"])

    def _on_endpoint_registered(self, event: Event) -> None:
        if not event.cache_synced:
            self.refresh_routes()
        if event.payload.get("address_changed"):
            self._data_plane.close_connection(self._event_lid(event))

    def _on_endpoint_deregistered(self, event: Event) -> None:
        lid = self._event_lid(event)
        self.route_table.remove(lid)
        self._data_plane.close_connection(lid)

    def _on_route_updated(self, event: Event) -> None:
        lid = self._event_lid(event)
        adjacent = abs(lid.stage_idx - self.lid.stage_idx) == 1
        sibling = lid.stage_idx == self.lid.stage_idx and lid.replica_idx != self.lid.replica_idx
        if adjacent or sibling:
            self._data_plane.close_connection(lid)
        if not event.cache_synced:
            self.refresh_routes()

    def _on_prepare_migration(self, event: Event) -> None:
        mid, new_address = event.payload["migration_id"], event.payload["new_address"]
        lid = self._event_lid(event)
        self._pending_migrations[mid] = {"lid": lid, "new_address": new_address, "state": "preparing"}
        if lid.model_name != self.lid.model_name:
            return
        self._shadow_manager.prepare_shadow(mid, lid, new_address)
        try:
            self.call("shadow_ready", {"migration_id": mid, "from_lid": self.lid.to_dict()})
        except Exception as e:  # noqa: BLE001
            logger.error("shadow_ready notify failed: %s", e)

    def _on_cutover_start(self, event: Event) -> None:
        pending = self._pending_migrations.get(event.payload["migration_id"])
        if pending is not None:
            pending["state"] = "cutting_over"

    def _on_cutover_complete(self, event: Event) -> None:
        mid = event.payload["migration_id"]
        self._shadow_manager.activate_shadow(mid)
        if not event.cache_synced:
            self.refresh_routes()
        self._pending_migrations.pop(mid, None)

    def _on_migration_failed(self, event: Event) -> None:
        mid = event.payload["migration_id"]
        self._shadow_manager.discard_shadow(mid)
        self._pending_migrations.pop(mid, None)

    def on_event(self, event_type: EventType, callback: Callable[[Event], None]) -> None:
        self._event_handlers.setdefault(event_type, []).append(callback)

    # ---------------------------------------------------------------- peers
    def get_peer_address(self, lid: LogicalEndpointID) -> Optional[str]:
        r = self.route_table.get(lid)
        return r.addresses[0] if r and r.addresses else None

    def get_pipeline_peers(self) -> List[RouteEntry]:
        return self.route_table.get_for_model(self.lid.model_name)

    def _neighbour(self, delta: int) -> Optional[RouteEntry]:
        want = self.lid.stage_idx + delta
        return next((r for r in self.get_pipeline_peers() if r.lid.stage_idx == want), None)

    def get_next_stage(self) -> Optional[RouteEntry]:
        return self._neighbour(+1)

    def get_prev_stage(self) -> Optional[RouteEntry]:
        return None if self.lid.stage_idx == 0 else self._neighbour(-1)

    def invalidate_peer_connection(self, lid: LogicalEndpointID) -> None:
        self._data_plane.close_connection(lid)
        self.refresh_routes()

    def report_failure(self, lid: LogicalEndpointID, reason: str = "reported") -> List[str]:
        try:
            return self.call("report_failure", {"lid": lid.to_dict(), "reason": reason}).get("failed", [])
        except Exception as e:  # noqa: BLE001
            logger.warning("report_failure failed: %s", e)
            return []

    def update_my_address(self, new_addresses: List[str]) -> bool:
        try:
            resp = self.call("update_route", {"lid": self.lid.to_dict(), "addresses": list(new_addresses)})
        except Exception as e:  # noqa: BLE001
            logger.error("address update failed: %s", e)
            return False
        if resp.get("success"):
            self.config.local_addresses = list(new_addresses)
            return True
        return False


def create_epc_client(model_name: str, stage_idx: int, front_router_api: str = "tcp://localhost:15555",
                      front_router_events: str = "tcp://localhost:15560", local_addresses: Optional[List[str]] = None,
                      **kwargs) -> EPCV2Client:
    return EPCV2Client(EPCV2ClientConfig(front_router_api=front_router_api,
                                         front_router_events=front_router_events, model_name=model_name,
                                         stage_idx=stage_idx, local_addresses=list(local_addresses or []),
                                         **kwargs))

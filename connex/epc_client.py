"""EPC v2 client: an engine's connection to the front router.

Registration, a fixed-rate heartbeat on its *own* self-healing REQ channel
(so a slow route query never delays liveness), an event subscriber that keeps
a model-scoped route cache current incrementally by event ``seq`` (a gap or
a heartbeat showing the router ahead -> one full refresh), cheap
stage-scoped peer queries, migration shadow handling and address updates.
Semantics follow the reference's ``connex/epc_client.py`` (``:142-1303``).

``serving_routes`` is the group rule: an ungrouped route serves; a group
(``group_size`` > 1) serves through its shard 0, and only while all its
shards are present.
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
    raw = os.environ.get(name)
    if not raw:
        return default
    try:
        return float(raw)
    except ValueError:
        return default


@dataclass
class RouteEntry:
    """Client view of a route (no timestamps / metadata besides the group)."""

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
                pass
        return cls(lid=LogicalEndpointID.from_dict(d["lid"]), addresses=list(d.get("addresses") or []),
                   capabilities=caps, epoch=int(d.get("epoch", 0)),
                   state=RouteState(int(d.get("state", RouteState.ACTIVE))),
                   group_size=int(d.get("group_size") or (d.get("metadata") or {}).get("group_size") or 1))


def serving_routes(routes: List[RouteEntry]) -> List[RouteEntry]:
    members: Dict[tuple, set] = {}
    for r in routes:
        if r.group_size > 1:
            members.setdefault((r.lid.model_name, r.lid.stage_idx, r.lid.replica_idx), set()).add(r.lid.shard_idx)
    out = []
    for r in routes:
        if r.group_size <= 1:
            out.append(r)
        elif r.lid.shard_idx == 0 and members[(r.lid.model_name, r.lid.stage_idx, r.lid.replica_idx)] \
                >= set(range(r.group_size)):
            out.append(r)
    return out


@dataclass
class Event(_RouterEvent):
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


class RouteTableCache:
    """Model-scoped local copy of the router's route table."""

    def __init__(self):
        self._routes: Dict[str, RouteEntry] = {}
        self._epoch = 0
        self._lock = threading.RLock()
        self._callbacks: List[Callable[[RouteEntry], None]] = []

    @property
    def epoch(self) -> int:
        with self._lock:
            return self._epoch

    def update_from_list(self, routes: List[Dict[str, Any]], epoch: int) -> None:
        with self._lock:
            self._routes = {}
            for d in routes:
                r = RouteEntry.from_dict(d)
                self._routes[r.lid.to_key()] = r
            self._epoch = epoch

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
            out = serving_routes([r for r in self._routes.values()
                                  if r.lid.model_name == model_name and r.lid.stage_idx == stage_idx])
        return sorted(out, key=lambda r: (r.lid.shard_idx, r.lid.replica_idx))

    def update_single(self, route: RouteEntry, epoch: int) -> None:
        with self._lock:
            self._routes[route.lid.to_key()] = route
            self._epoch = max(self._epoch, epoch)
            cbs = list(self._callbacks)
        for cb in cbs:
            try:
                cb(route)
            except Exception as e:
                logger.error("route callback failed: %s", e)

    def upsert(self, route: RouteEntry, epoch: int = 0) -> None:
        with self._lock:
            self._routes[route.lid.to_key()] = route
            self._epoch = max(self._epoch, epoch)

    def remove(self, lid: LogicalEndpointID) -> None:
        with self._lock:
            self._routes.pop(lid.to_key(), None)

    def set_state(self, lid: LogicalEndpointID, state: RouteState) -> bool:
        with self._lock:
            r = self._routes.get(lid.to_key())
            if r is None:
                return False
            r.state = state
            return True

    def replace_stage(self, model_name: str, stage_idx: int, routes: List[RouteEntry], epoch: int) -> None:
        with self._lock:
            for k in [k for k, r in self._routes.items()
                      if r.lid.model_name == model_name and r.lid.stage_idx == stage_idx]:
                del self._routes[k]
            for r in routes:
                self._routes[r.lid.to_key()] = r
            self._epoch = max(self._epoch, epoch)

    def add_callback(self, callback: Callable[[RouteEntry], None]) -> None:
        self._callbacks.append(callback)


class DataPlaneManager:
    """Bookkeeping of per-(LID, address) data-plane connections."""

    def __init__(self, config: EPCV2ClientConfig):
        self._config = config
        self._conns: Dict[str, Dict[str, Any]] = {}
        self._lock = threading.Lock()

    def get_or_create_connection(self, lid: LogicalEndpointID, address: str) -> Dict[str, Any]:
        key = f"{lid.to_key()}@{address}"
        with self._lock:
            return self._conns.setdefault(key, {"lid": lid, "address": address, "created_at": time.time()})

    def close_connection(self, lid: LogicalEndpointID) -> None:
        with self._lock:
            for k in [k for k in self._conns if k.startswith(lid.to_key() + "@")]:
                del self._conns[k]

    def close_all(self) -> None:
        with self._lock:
            self._conns.clear()

    def connections(self) -> List[str]:
        with self._lock:
            return list(self._conns)


class ShadowConnectionManager:
    """Pre-built connections to a migration target (hitless cut-over)."""

    def __init__(self, data_plane: DataPlaneManager):
        self._dp = data_plane
        self._shadows: Dict[str, Dict[str, Any]] = {}
        self._lock = threading.Lock()

    def prepare_shadow(self, migration_id: str, lid: LogicalEndpointID, new_address: str) -> bool:
        with self._lock:
            if migration_id not in self._shadows:
                self._shadows[migration_id] = {"lid": lid, "new_address": new_address, "ready": True,
                                               "connection": self._dp.get_or_create_connection(lid, new_address),
                                               "created_at": time.time()}
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


class _ReqChannel:
    """Locked REQ socket that is recreated after any timeout or ZMQ error
    (a REQ socket that missed a reply is stuck in the wrong state)."""

    def __init__(self, context: zmq.Context, endpoint: str, timeout_ms: int, name: str):
        self._ctx, self._ep, self.timeout_ms, self._name = context, endpoint, int(timeout_ms), name
        self._lock = threading.Lock()
        self._sock: Optional[zmq.Socket] = None
        self._closed = False
        self.resets = 0

    def _ensure(self) -> zmq.Socket:
        if self._sock is None:
            s = self._ctx.socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
            s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
            s.connect(self._ep)
            self._sock = s
        return self._sock

    def _reset(self) -> None:
        if self._sock is not None:
            try:
                self._sock.close(linger=0)
            except Exception:
                pass
            self._sock = None
            self.resets += 1

    def call(self, request: Dict[str, Any], timeout_ms: Optional[int] = None) -> Dict[str, Any]:
        t = self.timeout_ms if timeout_ms is None else int(timeout_ms)
        with self._lock:
            if self._closed:
                raise RuntimeError("Not connected to Front Router")
            s = self._ensure()
            try:
                s.send_json(request)
                if not s.poll(t, zmq.POLLIN):
                    self._reset()
                    raise APITimeoutError(f"{self._name}: no reply to {request.get('method')!r} within {t} ms")
                return s.recv_json()
            except APITimeoutError:
                raise
            except zmq.ZMQError as e:
                self._reset()
                raise RuntimeError(f"{self._name}: ZMQ error: {e}") from e

    def close(self) -> None:
        with self._lock:
            self._closed = True
            if self._sock is not None:
                try:
                    self._sock.close(linger=0)
                except Exception:
                    pass
                self._sock = None


class EPCV2Client:
    def __init__(self, config: EPCV2ClientConfig):
        self.config = config
        self.lid = config.lid
        self._ctx: Optional[zmq.Context] = None
        self._api: Optional[_ReqChannel] = None
        self._hb: Optional[_ReqChannel] = None
        self._sub: Optional[zmq.Socket] = None
        self.route_table = RouteTableCache()
        self._data_plane = DataPlaneManager(config)
        self._shadow_manager = ShadowConnectionManager(self._data_plane)
        self._registered = False
        self._running = False
        self._local_epoch = 0
        self._stop_event = threading.Event()
        self._sync_lock = threading.RLock()
        self._last_seq: Optional[int] = None
        self._needs_full_refresh = False
        self._hb_seen_seq: Optional[int] = None
        self._stage_query_supported = True
        self.stats: Dict[str, int] = {"full_refreshes": 0, "stage_queries": 0, "incremental_applied": 0,
                                      "seq_gaps": 0, "heartbeat_failures": 0}
        self._heartbeat_thread: Optional[threading.Thread] = None
        self._event_thread: Optional[threading.Thread] = None
        self._event_handlers: Dict[EventType, List[Callable[[Event], None]]] = {}
        self._pending_migrations: Dict[str, Dict[str, Any]] = {}

    # ---------------------------------------------------------- lifecycle
    def _heartbeat_timeout_ms(self) -> int:
        if self.config.heartbeat_timeout_ms:
            return int(self.config.heartbeat_timeout_ms)
        return int(min(self.config.api_timeout_ms, max(500, self.config.heartbeat_interval_s * 1000)))

    def start(self) -> bool:
        try:
            self._ctx = zmq.Context()
            self._stop_event.clear()
            self._api = _ReqChannel(self._ctx, self.config.front_router_api, self.config.api_timeout_ms, "epc-api")
            self._hb = _ReqChannel(self._ctx, self.config.front_router_api, self._heartbeat_timeout_ms(),
                                   "epc-heartbeat")
            self._sub = self._ctx.socket(zmq.SUB)
            self._sub.setsockopt(zmq.LINGER, 0)
            self._sub.connect(self.config.front_router_events)
            self._sub.setsockopt_string(zmq.SUBSCRIBE, "connex.")
            self._running = True
            if not self._register():
                self.stop()
                return False
            self._event_thread = threading.Thread(target=self._event_loop, daemon=True,
                                                  name=f"epc-events-{self.lid.stage_idx}")
            self._event_thread.start()
            self._heartbeat_thread = threading.Thread(target=self._heartbeat_loop, daemon=True,
                                                      name=f"epc-heartbeat-{self.lid.stage_idx}")
            self._heartbeat_thread.start()
            return True
        except Exception as e:
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
        """Stop without deregistering (as if the process died): the router only
        learns through the missed lease.  Used by failure tests."""
        self.stop(deregister=False)

    # ---------------------------------------------------------------- api
    def _call_api(self, method: str, params: Dict[str, Any], channel: Optional[_ReqChannel] = None,
                  timeout_ms: Optional[int] = None) -> Dict[str, Any]:
        ch = channel if channel is not None else self._api
        if ch is None:
            raise RuntimeError("Not connected to Front Router")
        resp = ch.call({"method": method, "params": params}, timeout_ms)
        if "error" in resp:
            raise RuntimeError(f"API error: {resp['error']}")
        return resp

    def _register(self, channel: Optional[_ReqChannel] = None) -> bool:
        params = {"lid": self.lid.to_dict(), "addresses": list(self.config.local_addresses),
                  "capabilities": [int(c) for c in self.config.capabilities]}
        if self.config.group_size > 1:
            params["group_size"] = int(self.config.group_size)
        try:
            resp = self._call_api("register", params, channel=channel)
        except Exception as e:
            logger.error("registration failed: %s", e)
            return False
        if not resp.get("success"):
            return False
        self._local_epoch = resp.get("epoch", 0)
        self._registered = True
        self._apply_snapshot(resp.get("route_table", []), self._local_epoch, resp.get("seq"))
        return True

    def _deregister(self) -> None:
        try:
            self._call_api("deregister", {"lid": self.lid.to_dict()})
            self._registered = False
        except Exception as e:
            logger.warning("deregistration failed: %s", e)

    def _send_heartbeat(self) -> bool:
        try:
            resp = self._call_api("heartbeat", {"lid": self.lid.to_dict()}, channel=self._hb)
        except Exception as e:
            self.stats["heartbeat_failures"] += 1
            logger.debug("heartbeat failed: %s", e)
            return False
        self._local_epoch = max(self._local_epoch, resp.get("epoch", 0))
        self._check_seq_from_heartbeat(resp.get("seq"))
        ok = bool(resp.get("success", False))
        if not ok and self._running:
            logger.warning("heartbeat rejected (unknown endpoint): re-registering")
            return self._register(channel=self._hb)
        return ok

    def _check_seq_from_heartbeat(self, server_seq: Optional[int]) -> None:
        """If the router's seq seen one heartbeat ago is still ahead of what
        this client processed, events were lost: schedule a full refresh."""
        if server_seq is None:
            return
        with self._sync_lock:
            prev, self._hb_seen_seq = self._hb_seen_seq, server_seq
            if prev is not None and (self._last_seq is None or self._last_seq < prev):
                self._needs_full_refresh = True

    def _apply_snapshot(self, routes, epoch: int, seq: Optional[int]) -> bool:
        with self._sync_lock:
            if seq is not None and self._last_seq is not None and seq < self._last_seq \
                    and not self._needs_full_refresh:
                return False
            self.route_table.update_from_list(routes, epoch)
            if seq is not None:
                self._last_seq = seq
                self._needs_full_refresh = False
            return True

    def refresh_routes(self) -> List[RouteEntry]:
        try:
            resp = self._call_api("get_routes", {"model_name": self.lid.model_name})
        except Exception as e:
            logger.error("route refresh failed: %s", e)
            return []
        epoch = resp.get("epoch", self._local_epoch)
        self._apply_snapshot(resp.get("routes", []), epoch, resp.get("seq"))
        self._local_epoch = max(self._local_epoch, epoch)
        self.stats["full_refreshes"] += 1
        return self.route_table.get_all()

    def cache_in_sync(self) -> bool:
        with self._sync_lock:
            return (self._last_seq is not None and not self._needs_full_refresh
                    and self._event_thread is not None and self._event_thread.is_alive())

    def query_stage_routes(self, stage_idx: int) -> Optional[List[RouteEntry]]:
        model = self.lid.model_name
        try:
            resp = None
            if self._stage_query_supported:
                try:
                    resp = self._call_api("get_stage_routes", {"model_name": model, "stage_idx": int(stage_idx)})
                except RuntimeError as e:
                    if "Unknown method" not in str(e):
                        raise
                    self._stage_query_supported = False
            if resp is None:
                self.refresh_routes()
                return self.route_table.get_for_stage(model, int(stage_idx))
            self.stats["stage_queries"] += 1
            entries = [RouteEntry.from_dict(r) for r in resp.get("routes", [])]
            seq = resp.get("seq")
            with self._sync_lock:
                if not (seq is not None and self._last_seq is not None and seq < self._last_seq
                        and not self._needs_full_refresh):
                    self.route_table.replace_stage(model, int(stage_idx), entries,
                                                   resp.get("epoch", self._local_epoch))
            return sorted(serving_routes(entries), key=lambda r: (r.lid.shard_idx, r.lid.replica_idx))
        except Exception as e:
            logger.warning("stage %s route query failed: %s", stage_idx, e)
            return None

    def get_stage_peers(self, stage_idx: int, refresh: str = "auto") -> List[RouteEntry]:
        """Routes of a stage: ``never`` = cache only; ``auto`` = cache while it
        is event-synced, else a stage query; ``always`` = stage query."""
        if refresh not in ("never", "auto", "always"):
            raise ValueError(f"invalid refresh mode: {refresh!r}")
        if refresh == "always" or (refresh == "auto" and not self.cache_in_sync()):
            res = self.query_stage_routes(stage_idx)
            if res is not None:
                return res
        return self.route_table.get_for_stage(self.lid.model_name, int(stage_idx))

    # ------------------------------------------------------------- events
    def _event_loop(self) -> None:
        last_retry = 0.0
        while self._running:
            try:
                if self._sub.poll(timeout=200):
                    _topic, data = self._sub.recv_multipart()
                    self._handle_event(Event.deserialize(data))
                elif self._needs_full_refresh and self._running and time.monotonic() - last_retry > 1.0:
                    last_retry = time.monotonic()
                    self.refresh_routes()
            except Exception as e:
                if self._running:
                    logger.error("event loop error: %s", e)

    def _sync_cache_from_event(self, event: Event) -> bool:
        if event.seq is None:
            return False
        with self._sync_lock:
            last = self._last_seq
            if last is not None and event.seq <= last and not self._needs_full_refresh:
                return True
            gap = last is None or self._needs_full_refresh or event.seq != last + 1
        if gap:
            with self._sync_lock:
                self.stats["seq_gaps"] += 1
                self._needs_full_refresh = True
            self.refresh_routes()
            with self._sync_lock:
                if self._needs_full_refresh or self._last_seq is None:
                    return False
                if event.seq <= self._last_seq:
                    return True
                if event.seq != self._last_seq + 1:
                    self._needs_full_refresh = True
                    return False
        with self._sync_lock:
            if self._apply_event_locked(event):
                self._last_seq = event.seq
                self.stats["incremental_applied"] += 1
                return True
            self._needs_full_refresh = True
            return False

    def _apply_event_locked(self, event: Event) -> bool:
        p = event.payload or {}
        if p.get("lid") is None:
            return True
        lid = LogicalEndpointID.from_dict(p["lid"])
        if lid.model_name != self.lid.model_name:
            return True
        t = event.type
        if t in (EventType.ENDPOINT_REGISTERED, EventType.ROUTE_UPDATED, EventType.CUTOVER_COMPLETE):
            if "route" not in p:
                return False
            self.route_table.upsert(RouteEntry.from_dict(p["route"]), event.epoch)
        elif t == EventType.ENDPOINT_DEREGISTERED:
            self.route_table.remove(lid)
        elif t == EventType.ENDPOINT_UNHEALTHY:
            self.route_table.set_state(lid, RouteState.UNHEALTHY)
        elif t == EventType.PREPARE_MIGRATION:
            self.route_table.set_state(lid, RouteState.MIGRATING)
        elif t == EventType.MIGRATION_FAILED:
            self.route_table.set_state(lid, RouteState.ACTIVE)
        return True

    def _handle_event(self, event: Event) -> None:
        self._local_epoch = max(self._local_epoch, event.epoch)
        try:
            event.cache_synced = self._sync_cache_from_event(event)
        except Exception as e:
            logger.error("route cache sync error: %s", e)
            event.cache_synced = False
        if event.source_lid == self.lid.to_key():
            return
        builtin = {EventType.ENDPOINT_REGISTERED: self._on_endpoint_registered,
                   EventType.ENDPOINT_DEREGISTERED: self._on_endpoint_deregistered,
                   EventType.PREPARE_MIGRATION: self._on_prepare_migration,
                   EventType.CUTOVER_START: self._on_cutover_start,
                   EventType.CUTOVER_COMPLETE: self._on_cutover_complete,
                   EventType.MIGRATION_FAILED: self._on_migration_failed,
                   EventType.ROUTE_UPDATED: self._on_route_updated}.get(event.type)
        for h in ([builtin] if builtin else []) + list(self._event_handlers.get(event.type, [])):
            try:
                h(event)
            except Exception as e:
                logger.error("event handler error: %s", e)

    def _on_endpoint_registered(self, event: Event) -> None:
        if not event.cache_synced:
            self.refresh_routes()
        if event.payload.get("address_changed"):
            self._data_plane.close_connection(LogicalEndpointID.from_dict(event.payload["lid"]))

    def _on_endpoint_deregistered(self, event: Event) -> None:
        lid = LogicalEndpointID.from_dict(event.payload["lid"])
        self.route_table.remove(lid)
        self._data_plane.close_connection(lid)

    def _on_route_updated(self, event: Event) -> None:
        lid = LogicalEndpointID.from_dict(event.payload["lid"])
        neighbour = abs(lid.stage_idx - self.lid.stage_idx) == 1 or \
            (lid.stage_idx == self.lid.stage_idx and lid.replica_idx != self.lid.replica_idx)
        if neighbour:
            self._data_plane.close_connection(lid)
        if not event.cache_synced:
            self.refresh_routes()

    def _on_prepare_migration(self, event: Event) -> None:
        mid = event.payload["migration_id"]
        lid = LogicalEndpointID.from_dict(event.payload["lid"])
        self._pending_migrations[mid] = {"lid": lid, "new_address": event.payload["new_address"],
                                         "state": "preparing"}
        if lid.model_name == self.lid.model_name:
            self._shadow_manager.prepare_shadow(mid, lid, event.payload["new_address"])
            try:
                self._call_api("shadow_ready", {"migration_id": mid, "from_lid": self.lid.to_dict()})
            except Exception as e:
                logger.error("shadow_ready notify failed: %s", e)

    def _on_cutover_start(self, event: Event) -> None:
        m = self._pending_migrations.get(event.payload["migration_id"])
        if m is not None:
            m["state"] = "cutting_over"

    def _on_cutover_complete(self, event: Event) -> None:
        self._shadow_manager.activate_shadow(event.payload["migration_id"])
        if not event.cache_synced:
            self.refresh_routes()
        self._pending_migrations.pop(event.payload["migration_id"], None)

    def _on_migration_failed(self, event: Event) -> None:
        self._shadow_manager.discard_shadow(event.payload["migration_id"])
        self._pending_migrations.pop(event.payload["migration_id"], None)

    def on_event(self, event_type: EventType, callback: Callable[[Event], None]) -> None:
        self._event_handlers.setdefault(event_type, []).append(callback)

    def _heartbeat_loop(self) -> None:
        interval = max(0.01, float(self.config.heartbeat_interval_s))
        nxt = time.monotonic()
        while self._running:
            if self._registered:
                self._send_heartbeat()
            nxt += interval
            delay = nxt - time.monotonic()
            if delay < 0:
                nxt, delay = time.monotonic(), 0
            if self._stop_event.wait(delay):
                break

    # -------------------------------------------------------------- peers
    def get_peer_address(self, lid: LogicalEndpointID) -> Optional[str]:
        r = self.route_table.get(lid)
        return r.addresses[0] if r and r.addresses else None

    def get_pipeline_peers(self) -> List[RouteEntry]:
        return self.route_table.get_for_model(self.lid.model_name)

    def get_next_stage(self) -> Optional[RouteEntry]:
        return next((r for r in self.get_pipeline_peers() if r.lid.stage_idx == self.lid.stage_idx + 1), None)

    def get_prev_stage(self) -> Optional[RouteEntry]:
        if self.lid.stage_idx == 0:
            return None
        return next((r for r in self.get_pipeline_peers() if r.lid.stage_idx == self.lid.stage_idx - 1), None)

    def invalidate_peer_connection(self, lid: LogicalEndpointID) -> None:
        self._data_plane.close_connection(lid)
        self.refresh_routes()

    def report_failure(self, lid: LogicalEndpointID, reason: str = "reported") -> List[str]:
        try:
            return self._call_api("report_failure", {"lid": lid.to_dict(), "reason": reason}).get("failed", [])
        except Exception as e:
            logger.warning("report_failure failed: %s", e)
            return []

    def update_my_address(self, new_addresses: List[str]) -> bool:
        try:
            resp = self._call_api("update_route", {"lid": self.lid.to_dict(), "addresses": list(new_addresses)})
        except Exception as e:
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

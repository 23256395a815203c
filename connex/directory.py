"""Directory client: LID -> physical address registry over ZeroMQ.

Wire protocol (msgpack maps over a DEALER socket, one request in flight per
socket; events as msgpack maps on the directory's PUB socket):

* ``{"type": "register", "event": JOIN|MIGRATE|LEAVE, "endpoint": {...}}``
* ``{"type": "lookup", "lid": [...], "epoch": e}``
* ``{"type": "list_stage", "model": m, "stage": s}``
* ``{"type": "request_assignment", "source_stage", "target_stage", "direction", "model"}``
* ``{"type": "heartbeat", "lid": [...]}`` / ``{"type": "report_failure", "lid": [...]}``
* ``{"type": "info"}`` -> ``{"event_address", "lease_s", "epoch"}``
* events: ``{"event", "endpoint", "epoch", "reason"}``

The same messages as ``connex/directory.py`` / ``connex/directory_server.py``
of the reference (``directory.py:218-625``), so either side interoperates.
Replies that arrive after a request timed out are drained before the next
request so a stale answer is never mistaken for the current one.
"""
from __future__ import annotations

import logging
import threading
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Callable, Optional

import msgpack
import zmq

logger = logging.getLogger("connex.directory")


class MembershipEvent(Enum):
    JOIN = "JOIN"
    LEAVE = "LEAVE"
    MIGRATE = "MIGRATE"
    PREPARE = "PREPARE"
    CUTOVER = "CUTOVER"
    FINALIZE = "FINALIZE"


class TransportCapability(Enum):
    UCX_RDMA = "ucx_rdma"
    UCX_TCP = "ucx_tcp"
    UCX_SHM = "ucx_shm"
    ZEROMQ = "zeromq"
    NVLINK = "nvlink"


def _caps_from(values) -> list:
    out = []
    for c in values or []:
        try:
            out.append(TransportCapability(c))
        except ValueError:
            logger.debug("unknown transport capability %r ignored", c)
    return out


@dataclass
class EndpointInfo:
    """Where a LID currently lives and what it can speak."""

    lid: tuple
    addresses: list
    transport_caps: list
    epoch: int = 0
    priority_classes: list = field(default_factory=lambda: ["token", "control"])
    metadata: dict = field(default_factory=dict)
    last_heartbeat: float = 0.0
    state: str = "active"

    model = property(lambda self: self.lid[0])
    stage = property(lambda self: self.lid[1])
    shard = property(lambda self: self.lid[2])
    replica = property(lambda self: self.lid[3])

    @property
    def primary_address(self) -> str:
        return self.addresses[0] if self.addresses else ""

    def to_dict(self) -> dict:
        return {"lid": self.lid, "addresses": self.addresses,
                "transport_caps": [c.value for c in self.transport_caps], "epoch": self.epoch,
                "priority_classes": self.priority_classes, "metadata": self.metadata,
                "state": self.state}

    @classmethod
    def from_dict(cls, d: dict) -> "EndpointInfo":
        return cls(lid=tuple(d["lid"]), addresses=list(d.get("addresses") or []),
                   transport_caps=_caps_from(d.get("transport_caps")), epoch=d.get("epoch", 0),
                   priority_classes=d.get("priority_classes", ["token", "control"]),
                   metadata=d.get("metadata", {}) or {}, state=d.get("state", "active"))


def _pack(msg: dict) -> bytes:
    return msgpack.packb(msg, use_bin_type=True)


def _unpack(data: bytes) -> dict:
    return msgpack.unpackb(data, raw=False)


def _drain(sock: Optional[zmq.Socket]) -> None:
    if sock is None:
        return
    while True:
        try:
            sock.recv(zmq.NOBLOCK)
        except zmq.Again:
            return


class DirectoryClient:
    """Registers one LID, looks others up, and delivers membership events."""

    def __init__(self, front_router_addr: str, model_name: str, stage_idx: int, shard_idx: int = 0,
                 replica_idx: int = 0, local_addresses: Optional[list] = None,
                 transport_caps: Optional[list] = None):
        self.front_router_addr = front_router_addr
        self.model_name = model_name
        self.stage_idx = stage_idx
        self.shard_idx = shard_idx
        self.replica_idx = replica_idx
        self.lid = (model_name, stage_idx, shard_idx, replica_idx)
        self.local_addresses = list(local_addresses or [])
        self.transport_caps = list(transport_caps or [TransportCapability.UCX_RDMA,
                                                      TransportCapability.UCX_TCP,
                                                      TransportCapability.ZEROMQ])
        self._epoch = 0
        self._epoch_lock = threading.Lock()
        self._endpoint_cache: dict = {}
        self._cache_lock = threading.RLock()
        self._event_handlers: list = []
        self._ctx = zmq.Context.instance()
        self._control_socket: Optional[zmq.Socket] = None
        self._control_lock = threading.Lock()
        self._sub_socket: Optional[zmq.Socket] = None
        self._running = False
        self._event_thread: Optional[threading.Thread] = None
        self._hb_thread: Optional[threading.Thread] = None
        self._hb_stop = threading.Event()
        self._registered: Optional[dict] = None

    # --------------------------------------------------------- lifecycle
    def start(self) -> None:
        if self._running:
            return
        self._running = True
        s = self._ctx.socket(zmq.DEALER)
        s.setsockopt(zmq.LINGER, 0)
        s.setsockopt_string(zmq.IDENTITY, "connex-{}-{}-{}-{}".format(*self.lid))
        s.connect(f"tcp://{self.front_router_addr}")
        self._control_socket = s

    def stop(self) -> None:
        self._running = False
        self._hb_stop.set()
        for th in (self._hb_thread, self._event_thread):
            if th is not None:
                th.join(timeout=2.0)
        self._hb_thread = self._event_thread = None
        for s in (self._control_socket, self._sub_socket):
            if s is not None:
                s.close()
        self._control_socket = self._sub_socket = None

    # -------------------------------------------------------- membership
    def _endpoint_msg(self, event: MembershipEvent, addresses: list, epoch: int, state: str) -> dict:
        return {"type": "register", "event": event.value,
                "endpoint": {"lid": self.lid, "addresses": addresses,
                             "transport_caps": [c.value for c in self.transport_caps],
                             "epoch": epoch, "state": state}}

    def register(self, addresses: Optional[list] = None) -> bool:
        addresses = addresses or self.local_addresses
        if not addresses:
            logger.warning("no addresses to register for %s", self.lid)
            return False
        ep = EndpointInfo(lid=self.lid, addresses=list(addresses), transport_caps=self.transport_caps,
                          epoch=self._epoch)
        req = {"type": "register", "event": MembershipEvent.JOIN.value, "endpoint": ep.to_dict()}
        resp = self._safe_call(req, 5000)
        if resp and resp.get("status") == "ok":
            self._registered = req
            with self._cache_lock:
                self._endpoint_cache[self.lid] = ep
            return True
        logger.error("registration of %s failed: %s", self.lid, resp)
        return False

    def notify_migration(self, new_addresses: list, target_epoch: int) -> bool:
        resp = self._safe_call(self._endpoint_msg(MembershipEvent.MIGRATE, list(new_addresses),
                                                  target_epoch, "migrating"), 5000)
        if resp and resp.get("status") == "ok":
            with self._epoch_lock:
                self._epoch = target_epoch
            return True
        return False

    def deregister(self) -> bool:
        resp = self._safe_call(self._endpoint_msg(MembershipEvent.LEAVE, [], self._epoch, "leaving"), 5000)
        if resp and resp.get("status") == "ok":
            self._registered = None
            self._hb_stop.set()
            self.invalidate_cache(self.lid)
            return True
        return False

    def report_failure(self, target_lid: tuple) -> bool:
        resp = self._safe_call({"type": "report_failure", "lid": list(target_lid)}, 2000)
        self.invalidate_cache(tuple(target_lid))
        return bool(resp and resp.get("status") == "ok")

    # ------------------------------------------------------------ lookup
    def lookup(self, target_lid: tuple) -> Optional[EndpointInfo]:
        target_lid = tuple(target_lid)
        with self._cache_lock:
            cached = self._endpoint_cache.get(target_lid)
            if cached is not None and cached.epoch >= self._epoch:
                return cached
        resp = self._safe_call({"type": "lookup", "lid": target_lid, "epoch": self._epoch}, 5000)
        if resp and resp.get("status") == "ok":
            ep = EndpointInfo.from_dict(resp["endpoint"])
            with self._cache_lock:
                self._endpoint_cache[target_lid] = ep
            return ep
        return None

    def lookup_stage(self, stage_idx: int) -> Optional[EndpointInfo]:
        return self.lookup((self.model_name, stage_idx, 0, 0))

    def list_stage(self, stage_idx: int) -> list:
        resp = self._safe_call({"type": "list_stage", "model": self.model_name, "stage": stage_idx}, 5000)
        if not resp or resp.get("status") != "ok":
            return []
        return [EndpointInfo.from_dict(e) for e in resp.get("endpoints", [])]

    def request_assignment(self, target_stage: int, direction: str) -> Optional[tuple]:
        resp = self._safe_call({"type": "request_assignment", "source_stage": self.stage_idx,
                                "target_stage": target_stage, "direction": direction,
                                "model": self.model_name}, 5000)
        if resp and resp.get("status") == "ok":
            return resp.get("endpoint", ""), resp.get("routing_key", "")
        return None

    # --------------------------------------------------------- liveness
    def start_heartbeat(self, interval_s: float = 0.5) -> None:
        """Renew this LID's lease; re-register if the directory evicted it."""
        if self._hb_thread is not None:
            return
        self._hb_stop.clear()
        self._hb_thread = threading.Thread(target=self._heartbeat_loop, args=(interval_s,), daemon=True,
                                           name=f"connex-dir-hb-{self.stage_idx}-{self.replica_idx}")
        self._hb_thread.start()

    def _heartbeat_loop(self, interval_s: float) -> None:
        sock = self._ctx.socket(zmq.DEALER)
        sock.setsockopt(zmq.LINGER, 0)
        sock.connect(f"tcp://{self.front_router_addr}")

        def call(msg):
            _drain(sock)
            sock.send(_pack(msg))
            return _unpack(sock.recv()) if sock.poll(int(interval_s * 2000)) else None

        try:
            while not self._hb_stop.is_set():
                reg = self._registered
                if reg is not None:
                    resp = call({"type": "heartbeat", "lid": list(self.lid)})
                    if resp and resp.get("status") == "not_found" and self._registered is not None:
                        logger.warning("%s was evicted; re-registering", self.lid)
                        call(reg)
                        call({"type": "heartbeat", "lid": list(self.lid)})
                self._hb_stop.wait(interval_s)
        finally:
            sock.close()

    # ------------------------------------------------------------ events
    def start_event_listener(self, event_address: Optional[str] = None) -> bool:
        """Deliver PUB membership events to ``subscribe_events`` handlers.
        Subscribe before snapshotting (``list_stage``) so no change is lost."""
        if self._event_thread is not None:
            return True
        if event_address is None:
            info = self._safe_call({"type": "info"}, 2000)
            if not info or info.get("status") != "ok" or not info.get("event_address"):
                return False
            host, port = info["event_address"].rsplit(":", 1)
            if host in ("0.0.0.0", "*"):
                host = self.front_router_addr.rsplit(":", 1)[0]
            event_address = f"{host}:{port}"
        sub = self._ctx.socket(zmq.SUB)
        sub.setsockopt(zmq.LINGER, 0)
        sub.setsockopt(zmq.SUBSCRIBE, b"")
        sub.connect(f"tcp://{event_address}")
        self._sub_socket = sub
        ready = threading.Event()
        self._event_thread = threading.Thread(target=self._event_loop, args=(ready,), daemon=True,
                                              name=f"connex-dir-events-{self.stage_idx}")
        self._event_thread.start()
        ready.wait(1.0)
        return True

    def _event_loop(self, ready: threading.Event) -> None:
        sock = self._sub_socket
        sock.poll(100)  # let the subscription settle before callers snapshot
        ready.set()
        while self._running:
            if not sock.poll(100):
                continue
            try:
                msg = _unpack(sock.recv())
                event = MembershipEvent(msg["event"])
                info = EndpointInfo.from_dict(msg["endpoint"])
            except Exception as e:  # malformed event
                logger.warning("bad directory event: %s", e)
                continue
            if msg.get("epoch") is not None:
                with self._epoch_lock:
                    self._epoch = max(self._epoch, msg["epoch"])
            if event == MembershipEvent.LEAVE:
                self.invalidate_cache(info.lid)
            for h in list(self._event_handlers):
                try:
                    h(event, info)
                except Exception:
                    logger.exception("directory event handler failed")

    def subscribe_events(self, handler: Callable) -> None:
        self._event_handlers.append(handler)

    # ------------------------------------------------------------- epoch
    def get_current_epoch(self) -> int:
        with self._epoch_lock:
            return self._epoch

    def increment_epoch(self) -> int:
        with self._epoch_lock:
            self._epoch += 1
            return self._epoch

    def invalidate_cache(self, target_lid: Optional[tuple] = None) -> None:
        with self._cache_lock:
            if target_lid:
                self._endpoint_cache.pop(tuple(target_lid), None)
            else:
                self._endpoint_cache.clear()

    # ------------------------------------------------------------- wire
    def _safe_call(self, message: dict, timeout_ms: int) -> Optional[dict]:
        try:
            return self._control_call(message, timeout_ms)
        except Exception as e:
            logger.error("directory request %s failed: %s", message.get("type"), e)
            return None

    def _control_call(self, message: dict, timeout_ms: int = 5000) -> Optional[dict]:
        with self._control_lock:
            sock = self._control_socket
            if sock is None:
                return None
            _drain(sock)
            sock.send(_pack(message))
            if sock.poll(timeout_ms):
                return _unpack(sock.recv())
            return None

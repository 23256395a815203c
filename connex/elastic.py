"""ElasticPeerSet: directory membership turned into connected, routable peers.

Semantics (the reference's ``connex/elastic.py:49-261``):

* JOIN / MIGRATE -- the new address is connected on a background pool and
  becomes routable only once connected; a connect that finishes after the
  LID left or moved again is discarded (stale-connect guard); a migrated
  LID's old endpoint is drained, then closed.
* LEAVE (deregister / lease expiry / reported failure) -- unroutable at once;
  the endpoint closes after ``drain_grace_s`` unless the same endpoint is in
  use again (transports cache endpoints per address, so a same-address
  rejoin can share it).
* send failure -- ``mark_failed``: drop locally, ``report_failure`` to the
  directory (which tells every other sender), close.
* membership comes from directory push events, else from polling
  ``list_stage`` every ``poll_s`` on a private client.

``transport`` needs ``connect_sync(host, port)``, ``send_sync(ep, data, tag)``
and ``close_endpoint(ep)``; :class:`ZmqTransport` is the CPU one and
:class:`connex_b200.engine.CxEngineTransport` the native one.
"""
from __future__ import annotations

import logging
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Optional

from connex.directory import DirectoryClient, EndpointInfo, MembershipEvent

logger = logging.getLogger("connex.elastic")


class ElasticPeerSet:
    def __init__(self, directory: DirectoryClient, transport: Any, stage_idx: int,
                 drain_grace_s: float = 1.0, poll_s: float = 0.1, connect_workers: int = 4):
        self.directory = directory
        self.transport = transport
        self.stage_idx = stage_idx
        self.drain_grace_s = drain_grace_s
        self.poll_s = poll_s
        self._lock = threading.Lock()
        self._cv = threading.Condition(self._lock)
        self._ready: dict = {}    # lid -> (endpoint, address)
        self._wanted: dict = {}   # lid -> address we should be connected to
        self._order: list = []    # routable lids, sorted
        self._rr = 0
        self._pool = ThreadPoolExecutor(max_workers=connect_workers, thread_name_prefix="connex-peer")
        self._stop = threading.Event()
        self._push = False
        self._closed_on_stop: list = []
        self.stats = {"connects": 0, "connect_ms_total": 0.0, "failures": 0, "leaves": 0}

    # ---------------------------------------------------------- lifecycle
    def start(self) -> None:
        self.directory.subscribe_events(self._on_event)
        self._push = self.directory.start_event_listener()
        self._sync(self.directory.list_stage(self.stage_idx))  # snapshot after subscribing
        if not self._push:
            threading.Thread(target=self._poll_loop, daemon=True, name="connex-peer-poll").start()

    def stop(self) -> None:
        self._stop.set()
        with self._lock:
            eps = [ep for ep, _ in self._ready.values()]
            self._ready.clear()
            self._wanted.clear()
            self._order = []
            self._closed_on_stop = eps
        for ep in eps:
            self._close(ep)
        self._pool.shutdown(wait=False)

    # -------------------------------------------------------------- query
    def peers(self) -> list:
        with self._lock:
            return list(self._order)

    def wait_ready(self, n: int = 1, timeout: float = 30.0) -> bool:
        deadline = time.monotonic() + timeout
        with self._cv:
            while len(self._order) < n:
                left = deadline - time.monotonic()
                if left <= 0:
                    return False
                self._cv.wait(left)
            return True

    def pick(self) -> Optional[tuple]:
        with self._lock:
            if not self._order:
                return None
            lid = self._order[self._rr % len(self._order)]
            self._rr += 1
            return lid

    def endpoint(self, lid: tuple) -> Optional[Any]:
        with self._lock:
            e = self._ready.get(lid)
            return e[0] if e else None

    # --------------------------------------------------------------- data
    def send(self, lid: tuple, data: Any, tag: int = 0) -> None:
        ep = self.endpoint(lid)
        if ep is None:
            raise KeyError(f"peer {lid} is not routable")
        try:
            self.transport.send_sync(ep, data, tag)
        except Exception:
            self.mark_failed(lid)
            raise

    def mark_failed(self, lid: tuple) -> None:
        with self._lock:
            entry = self._ready.pop(lid, None)
            self._wanted.pop(lid, None)
            self._reorder()
        self.stats["failures"] += 1
        logger.warning("peer %s failed: removed and reported", lid)
        self.directory.report_failure(lid)
        if entry is not None:
            try:
                self._pool.submit(self._close, entry[0])
            except RuntimeError:
                self._close(entry[0])

    # ----------------------------------------------------------- internal
    def _reorder(self) -> None:  # lock held
        self._order = sorted(self._ready)
        self._cv.notify_all()

    def _on_event(self, event: MembershipEvent, info: EndpointInfo) -> None:
        if info.stage != self.stage_idx or info.model != self.directory.model_name:
            return
        if event == MembershipEvent.LEAVE:
            self._remove(info.lid)
        elif info.addresses:
            self._want(info.lid, info.primary_address)

    def _sync(self, members: list) -> None:
        current = {m.lid: m.primary_address for m in members if m.addresses}
        with self._lock:
            gone = [l for l in self._wanted if l not in current]
        for lid in gone:
            self._remove(lid)
        for lid, addr in current.items():
            self._want(lid, addr)

    def _poll_loop(self) -> None:
        client = DirectoryClient(self.directory.front_router_addr, self.directory.model_name,
                                 stage_idx=-1, replica_idx=id(self) & 0xFFFF)
        client.start()
        try:
            while not self._stop.wait(self.poll_s):
                self._sync(client.list_stage(self.stage_idx))
        finally:
            client.stop()

    def _want(self, lid: tuple, addr: str) -> None:
        with self._lock:
            if self._stop.is_set() or self._wanted.get(lid) == addr:
                return
            self._wanted[lid] = addr
        try:
            self._pool.submit(self._connect, lid, addr)
        except RuntimeError:
            with self._lock:
                if self._wanted.get(lid) == addr:
                    del self._wanted[lid]

    def _connect(self, lid: tuple, addr: str) -> None:
        host, port = addr.rsplit(":", 1)
        t0 = time.monotonic()
        try:
            ep = self.transport.connect_sync(host, int(port))
        except Exception as e:
            logger.warning("connect to %s at %s failed: %s", lid, addr, e)
            with self._lock:
                if self._wanted.get(lid) == addr:
                    del self._wanted[lid]
            return
        old = None
        with self._lock:
            stale = self._wanted.get(lid) != addr
            if not stale:
                old = self._ready.get(lid)
                self._ready[lid] = (ep, addr)
                self._reorder()
        if stale:
            self._close(ep)
            return
        dt = (time.monotonic() - t0) * 1000
        self.stats["connects"] += 1
        self.stats["connect_ms_total"] += dt
        if old is not None and old[0] is not ep:
            self._close_later(old[0])

    def _remove(self, lid: tuple) -> None:
        with self._lock:
            self._wanted.pop(lid, None)
            entry = self._ready.pop(lid, None)
            self._reorder()
        if entry is not None:
            self.stats["leaves"] += 1
            self._close_later(entry[0])

    def _close_later(self, ep: Any) -> None:
        def run():
            with self._lock:
                in_use = any(e is ep for e, _ in self._ready.values())
                closed = any(e is ep for e in self._closed_on_stop)
            if not in_use and not closed:
                self._close(ep)
        t = threading.Timer(self.drain_grace_s, run)
        t.daemon = True
        t.start()

    def _close(self, ep: Any) -> None:
        try:
            self.transport.close_endpoint(ep)
        except Exception as e:
            logger.debug("close_endpoint failed: %s", e)


class ZmqTransport:
    """CPU PUSH/PULL transport with endpoints cached by address."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0):
        import zmq
        self._zmq = zmq
        self._ctx = zmq.Context.instance()
        self._lock = threading.Lock()
        self._eps: dict = {}
        self._rx = self._ctx.socket(zmq.PULL)
        self._rx.setsockopt(zmq.LINGER, 0)
        if port:
            self._rx.bind(f"tcp://{host}:{port}")
            self.local_port = port
        else:
            self.local_port = self._rx.bind_to_random_port(f"tcp://{host}")

    def start_sync(self) -> None:
        pass

    def connect_sync(self, host: str, port: int) -> Any:
        with self._lock:
            ep = self._eps.get((host, port))
            if ep is None:
                ep = self._ctx.socket(self._zmq.PUSH)
                ep.setsockopt(self._zmq.LINGER, 0)
                ep.setsockopt(self._zmq.SNDTIMEO, 2000)
                ep.connect(f"tcp://{host}:{port}")
                self._eps[(host, port)] = ep
            return ep

    def send_sync(self, ep: Any, data: bytes, tag: int = 0) -> None:
        with self._lock:
            ep.send(data)

    def recv_sync(self, timeout_ms: int = 1000) -> Optional[bytes]:
        return self._rx.recv() if self._rx.poll(timeout_ms) else None

    def close_endpoint(self, ep: Any) -> bool:
        with self._lock:
            for k, v in list(self._eps.items()):
                if v is ep:
                    del self._eps[k]
        ep.close(0)
        return True

    def stop_sync(self) -> None:
        with self._lock:
            for ep in self._eps.values():
                ep.close(0)
            self._eps.clear()
        self._rx.close(0)

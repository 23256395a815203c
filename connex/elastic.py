"""ElasticPeerSet: directory membership turned into connected, routable peers.

Every LID of the watched stage has one :class:`_Peer` record holding the
address the directory lists for it, the endpoint currently connected (and
its address), and a *generation* number.  Every change of the listed
address and every removal bumps the generation; a connect attempt carries
the generation it was started for and its result is kept only if that is
still current, so a connect that completes after the LID left or moved
again is closed instead of routed (the stale-connect guard).

* JOIN / MIGRATE: the new address is connected on a worker pool; the LID
  becomes routable (or switches endpoint) only once connected.  An endpoint
  replaced by a migration is drained for ``drain_grace_s``, then closed.
* LEAVE (deregister, lease expiry, reported failure): unroutable at once;
  its endpoint is drained, then closed -- unless it is in use again by then
  (transports cache endpoints per address, so a same-address rejoin may
  share it).
* A failed send calls :meth:`ElasticPeerSet.mark_failed`: the peer is
  dropped here and reported to the directory, which tells every other
  sender.
* Membership arrives as directory push events; without them a private
  client polls ``list_stage`` every ``poll_s``.

Draining endpoints sit in one deadline queue served by a single reaper
thread.  ``transport`` needs ``connect_sync(host, port)``, ``send_sync(ep,
data, tag)`` and ``close_endpoint(ep)``: :class:`ZmqTransport` is the CPU
one, :class:`connex_b200.engine.CxEngineTransport` the native one.
Behavioural parity: ``connex/elastic.py:49-327`` of the reference.
"""
from __future__ import annotations

import heapq
import itertools
import logging
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

from connex.directory import DirectoryClient, EndpointInfo, MembershipEvent

logger = logging.getLogger("connex.elastic")


@dataclass
class _Peer:
    listed: Optional[str] = None       # the address the directory lists
    generation: int = 0
    endpoint: Any = None               # connected endpoint (routable when set)
    connected_to: Optional[str] = None


class _Reaper:
    """Closes endpoints once their drain deadline passes, unless ``keep(ep)``
    says they are in use again by then."""

    def __init__(self, close, keep):
        self._close, self._keep = close, keep
        self._heap: List[Tuple[float, int, Any]] = []
        self._cv = threading.Condition()
        self._seq = itertools.count()
        self._done = False
        self._thread = threading.Thread(target=self._run, daemon=True, name="connex-peer-drain")
        self._thread.start()

    def later(self, ep: Any, delay_s: float) -> None:
        with self._cv:
            heapq.heappush(self._heap, (time.monotonic() + delay_s, next(self._seq), ep))
            self._cv.notify()

    def stop(self) -> None:
        with self._cv:
            self._done = True
            self._cv.notify()

    def _run(self) -> None:
        while True:
            with self._cv:
                while not self._done and (not self._heap or self._heap[0][0] > time.monotonic()):
                    self._cv.wait(None if not self._heap else max(0.0, self._heap[0][0] - time.monotonic()))
                if self._done:
                    return
                _, _, ep = heapq.heappop(self._heap)
            if not self._keep(ep):
                self._close(ep)


class ElasticPeerSet:
    def __init__(self, directory: DirectoryClient, transport: Any, stage_idx: int,
                 drain_grace_s: float = 1.0, poll_s: float = 0.1, connect_workers: int = 4):
        self.directory = directory
        self.transport = transport
        self.stage_idx = stage_idx
        self.drain_grace_s = drain_grace_s
        self.poll_s = poll_s
        self._cv = threading.Condition()
        self._peers: Dict[tuple, _Peer] = {}
        self._gen = itertools.count(1)
        self._turn = itertools.count()
        self._pool = ThreadPoolExecutor(max_workers=connect_workers, thread_name_prefix="connex-peer")
        self._stopped = threading.Event()
        self._retired: List[Any] = []           # endpoints closed by stop()
        self._reaper = _Reaper(self._close, self._in_use)
        self.stats = {"connects": 0, "connect_ms_total": 0.0, "failures": 0, "leaves": 0}

    # ------------------------------------------------------------ lifecycle
    def start(self) -> None:
        self.directory.subscribe_events(self._on_event)
        pushed = self.directory.start_event_listener()
        self._reconcile(self.directory.list_stage(self.stage_idx))   # snapshot after subscribing
        if not pushed:
            threading.Thread(target=self._poll, daemon=True, name="connex-peer-poll").start()

    def stop(self) -> None:
        self._stopped.set()
        with self._cv:
            eps = [p.endpoint for p in self._peers.values() if p.endpoint is not None]
            self._peers.clear()
            self._retired = eps
            self._cv.notify_all()
        for ep in eps:
            self._close(ep)
        self._reaper.stop()
        self._pool.shutdown(wait=False)

    # ---------------------------------------------------------------- views
    def _routable(self) -> List[tuple]:          # lock held
        return sorted(lid for lid, p in self._peers.items() if p.endpoint is not None)

    def peers(self) -> list:
        with self._cv:
            return self._routable()

    def wait_ready(self, n: int = 1, timeout: float = 30.0) -> bool:
        with self._cv:
            return self._cv.wait_for(lambda: len(self._routable()) >= n, timeout)

    def pick(self) -> Optional[tuple]:
        """Round-robin over the routable peers."""
        with self._cv:
            ready = self._routable()
            return ready[next(self._turn) % len(ready)] if ready else None

    def endpoint(self, lid: tuple) -> Optional[Any]:
        with self._cv:
            p = self._peers.get(lid)
            return p.endpoint if p is not None else None

    def address(self, lid: tuple) -> Optional[str]:
        """The address ``lid``'s routable endpoint is connected to, or None."""
        with self._cv:
            p = self._peers.get(lid)
            return p.connected_to if p is not None and p.endpoint is not None else None

    def _in_use(self, ep: Any) -> bool:
        with self._cv:
            return any(p.endpoint is ep for p in self._peers.values()) or any(e is ep for e in self._retired)

    # ----------------------------------------------------------------- data
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
        """Drop a peer a send failed on and report it to the directory."""
        with self._cv:
            p = self._peers.pop(lid, None)
            self._cv.notify_all()
        self.stats["failures"] += 1
        logger.warning("peer %s failed: removed and reported", lid)
        self.directory.report_failure(lid)
        if p is not None and p.endpoint is not None:
            try:
                self._pool.submit(self._close, p.endpoint)
            except RuntimeError:          # pool already shut down
                self._close(p.endpoint)

    # ----------------------------------------------------------- membership
    def _on_event(self, event: MembershipEvent, info: EndpointInfo) -> None:
        if info.stage != self.stage_idx or info.model != self.directory.model_name:
            return
        if event == MembershipEvent.LEAVE:
            self._forget(info.lid)
        elif info.addresses:
            self._track(info.lid, info.primary_address)

    def _reconcile(self, members: list) -> None:
        listed = {m.lid: m.primary_address for m in members if m.addresses}
        with self._cv:
            gone = [lid for lid in self._peers if lid not in listed]
        for lid in gone:
            self._forget(lid)
        for lid, addr in listed.items():
            self._track(lid, addr)

    def _poll(self) -> None:
        client = DirectoryClient(self.directory.front_router_addr, self.directory.model_name,
                                 stage_idx=-1, replica_idx=id(self) & 0xFFFF)
        client.start()
        try:
            while not self._stopped.wait(self.poll_s):
                self._reconcile(client.list_stage(self.stage_idx))
        finally:
            client.stop()

    def _track(self, lid: tuple, addr: str) -> None:
        """The directory lists ``lid`` at ``addr``: connect unless already there."""
        with self._cv:
            if self._stopped.is_set():
                return
            p = self._peers.setdefault(lid, _Peer())
            if p.listed == addr:
                return
            p.listed, p.generation = addr, next(self._gen)
            gen = p.generation
        try:
            self._pool.submit(self._dial, lid, addr, gen)
        except RuntimeError:
            pass                              # stopping

    def _forget(self, lid: tuple) -> None:
        with self._cv:
            p = self._peers.pop(lid, None)
            self._cv.notify_all()
        if p is not None and p.endpoint is not None:
            self.stats["leaves"] += 1
            self._reaper.later(p.endpoint, self.drain_grace_s)

    def _dial(self, lid: tuple, addr: str, gen: int) -> None:
        host, port = addr.rsplit(":", 1)
        t0 = time.monotonic()
        try:
            ep = self.transport.connect_sync(host, int(port))
        except Exception as e:  # noqa: BLE001 - retried on the next listing of this address
            logger.warning("connect to %s at %s failed: %s", lid, addr, e)
            with self._cv:
                p = self._peers.get(lid)
                if p is not None and p.generation == gen:
                    p.listed = None
            return
        with self._cv:
            p = self._peers.get(lid)
            current = p is not None and p.generation == gen
            if current:
                replaced, p.endpoint, p.connected_to = p.endpoint, ep, addr
                self._cv.notify_all()
        if not current:
            self._close(ep)                    # the LID left or moved while we dialled
            return
        self.stats["connects"] += 1
        self.stats["connect_ms_total"] += (time.monotonic() - t0) * 1000
        if replaced is not None and replaced is not ep:
            self._reaper.later(replaced, self.drain_grace_s)

    def _close(self, ep: Any) -> None:
        try:
            self.transport.close_endpoint(ep)
        except Exception as e:  # noqa: BLE001
            logger.debug("close_endpoint failed: %s", e)


class ZmqTransport:
    """CPU transport: one PULL socket to receive on, one PUSH socket per
    destination address (shared by every LID at that address)."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0):
        import zmq
        self._zmq = zmq
        self._ctx = zmq.Context.instance()
        self._lock = threading.Lock()
        self._by_addr: Dict[Tuple[str, int], Any] = {}
        self._rx = self._ctx.socket(zmq.PULL)
        self._rx.setsockopt(zmq.LINGER, 0)
        if port:
            self._rx.bind(f"tcp://{host}:{port}")
            self.local_port = port
        else:
            self.local_port = self._rx.bind_to_random_port(f"tcp://{host}")

    def start_sync(self) -> None:
        return None

    def connect_sync(self, host: str, port: int) -> Any:
        with self._lock:
            sock = self._by_addr.get((host, port))
            if sock is None:
                sock = self._ctx.socket(self._zmq.PUSH)
                sock.setsockopt(self._zmq.LINGER, 0)
                sock.setsockopt(self._zmq.SNDTIMEO, 2000)
                sock.connect(f"tcp://{host}:{port}")
                self._by_addr[(host, port)] = sock
            return sock

    def send_sync(self, ep: Any, data: bytes, tag: int = 0) -> None:
        with self._lock:
            ep.send(data)

    def recv_sync(self, timeout_ms: int = 1000) -> Optional[bytes]:
        if not self._rx.poll(timeout_ms):
            return None
        return self._rx.recv()

    def close_endpoint(self, ep: Any) -> bool:
        with self._lock:
            self._by_addr = {k: s for k, s in self._by_addr.items() if s is not ep}
        ep.close(0)
        return True

    def stop_sync(self) -> None:
        with self._lock:
            socks, self._by_addr = list(self._by_addr.values()), {}
        for s in socks:
            s.close(0)
        self._rx.close(0)

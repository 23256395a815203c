"""In-memory directory service: ZeroMQ ROUTER for requests, PUB for events.

It speaks the msgpack protocol of :mod:`connex.directory` (wire parity with
``connex/directory_server.py:8-22`` of the reference):

* requests ``{"type": ...}`` -- ``register`` (event JOIN / MIGRATE / LEAVE),
  ``heartbeat``, ``report_failure``, ``lookup``, ``list_stage``,
  ``request_assignment``, ``info``; every reply carries ``status`` and the
  directory ``epoch``;
* events ``{"event", "endpoint", "epoch", "reason"}`` on the PUB socket, one
  per membership change, with reasons ``deregister`` / ``reported`` /
  ``expired`` for removals.

The membership itself is :class:`MembershipTable`, a plain object without
sockets: one epoch counter bumped by every change, the events not yet
published, and leases kept as a deadline heap (only members that have
heartbeated at least once hold a lease; each heartbeat pushes a new
deadline and older heap entries of that member are skipped when they
surface).  :class:`DirectoryServer` runs the table behind the two sockets.

    python -m connex.directory_server --bind 127.0.0.1:5555
"""
from __future__ import annotations

import argparse
import heapq
import logging
import threading
import time
from typing import Callable, Dict, List, Optional, Tuple

import msgpack
import zmq

from connex.directory import MembershipEvent

logger = logging.getLogger("connex.directory_server")

Key = Tuple


class MembershipTable:
    """Members by LID tuple, the directory epoch and the outgoing events."""

    def __init__(self, lease_s: float, clock: Callable[[], float] = time.monotonic):
        self.lease_s = lease_s
        self.clock = clock
        self.epoch = 0
        self.members: Dict[Key, dict] = {}
        self._deadline: Dict[Key, float] = {}          # current lease per heartbeating member
        self._heap: List[Tuple[float, Key]] = []
        self.pending: List[dict] = []

    # -------------------------------------------------------------- changes
    def _changed(self, event: str, endpoint: dict, reason: str) -> None:
        self.epoch += 1
        self.pending.append({"event": event, "endpoint": endpoint, "epoch": self.epoch, "reason": reason})

    def _renew(self, key: Key) -> None:
        due = self.clock() + self.lease_s
        self._deadline[key] = due
        heapq.heappush(self._heap, (due, key))

    def put(self, endpoint: dict, event: str) -> None:
        key = tuple(endpoint["lid"])
        self.members[key] = endpoint
        if key in self._deadline:           # re-registration of a heartbeating member renews its lease
            self._renew(key)
        self._changed(event, endpoint, "")

    def drop(self, key: Key, reason: str) -> bool:
        self._deadline.pop(key, None)
        endpoint = self.members.pop(key, None)
        if endpoint is None:
            return False
        self._changed(MembershipEvent.LEAVE.value, endpoint, reason)
        logger.info("LEAVE %s (%s, epoch %d)", key, reason, self.epoch)
        return True

    def heartbeat(self, key: Key) -> bool:
        if key not in self.members:
            return False
        self._renew(key)
        return True

    def expire(self) -> int:
        """Remove members whose lease ran out; returns how many."""
        now, n = self.clock(), 0
        while self._heap and self._heap[0][0] < now:
            due, key = heapq.heappop(self._heap)
            if self._deadline.get(key) == due:      # not renewed since this entry was pushed
                n += self.drop(key, "expired")
        return n

    def take_events(self) -> List[dict]:
        out, self.pending = self.pending, []
        return out

    # -------------------------------------------------------------- queries
    def stage(self, model: str, stage: int) -> List[Tuple[Key, dict]]:
        return sorted((k, ep) for k, ep in self.members.items() if k[0] == model and k[1] == stage)


class DirectoryServer:
    def __init__(self, bind_addr: str = "127.0.0.1:5555", event_bind_addr: Optional[str] = None,
                 lease_s: float = 2.0):
        self.bind_addr = bind_addr
        host, port = bind_addr.rsplit(":", 1)
        self.event_bind_addr = event_bind_addr or f"{host}:{int(port) + 1}"
        self.lease_s = lease_s
        self.table = MembershipTable(lease_s)
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._ready = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._bind_error: Optional[BaseException] = None
        self._ops = {"register": self._op_register, "heartbeat": self._op_heartbeat,
                     "report_failure": self._op_report_failure, "lookup": self._op_lookup,
                     "list_stage": self._op_list_stage, "request_assignment": self._op_assignment,
                     "info": self._op_info}

    @property
    def epoch(self) -> int:
        return self.table.epoch

    # ------------------------------------------------------------- lifecycle
    def start(self) -> None:
        self._thread = threading.Thread(target=self.serve_forever, daemon=True, name="connex-directory")
        self._thread.start()
        if not self._ready.wait(5) or self._bind_error is not None:
            raise RuntimeError(f"DirectoryServer failed to bind {self.bind_addr}: {self._bind_error}")

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(2)
            self._thread = None

    def members(self) -> dict:
        with self._lock:
            return dict(self.table.members)

    def _open(self):
        ctx = zmq.Context.instance()
        router, pub = ctx.socket(zmq.ROUTER), ctx.socket(zmq.PUB)
        for s in (router, pub):
            s.setsockopt(zmq.LINGER, 0)
        try:
            router.bind(f"tcp://{self.bind_addr}")
            pub.bind(f"tcp://{self.event_bind_addr}")
        except zmq.ZMQError as e:
            router.close()
            pub.close()
            raise e
        return router, pub

    def _answer(self, frames) -> bytes:
        try:
            reply = self.handle(msgpack.unpackb(frames[-1], raw=False))
        except Exception as e:  # noqa: BLE001 - a malformed request gets an error reply
            reply = {"status": "error", "error": str(e)}
        return msgpack.packb(reply, use_bin_type=True)

    def serve_forever(self) -> None:
        try:
            router, pub = self._open()
        except zmq.ZMQError as e:
            self._bind_error = e
            self._ready.set()
            return
        self._ready.set()
        poll_ms = int(1000 * min(0.05, self.lease_s / 4))
        try:
            while not self._stop.is_set():
                if router.poll(poll_ms):
                    # answer the whole burst, then publish its events together
                    while True:
                        try:
                            frames = router.recv_multipart(zmq.NOBLOCK)
                        except zmq.Again:
                            break
                        router.send_multipart([frames[0], self._answer(frames)])
                with self._lock:
                    self.table.expire()
                    events = self.table.take_events()
                for ev in events:
                    pub.send(msgpack.packb(ev, use_bin_type=True))
        finally:
            router.close()
            pub.close()

    # -------------------------------------------------------------- requests
    def handle(self, req: dict) -> dict:
        op = self._ops.get(req.get("type"))
        if op is None:
            return {"status": "error", "error": f"unknown request type {req.get('type')!r}"}
        with self._lock:
            return op(req)

    def _reply(self, ok: bool, **extra) -> dict:
        return {"status": "ok" if ok else "not_found", "epoch": self.table.epoch, **extra}

    def _op_register(self, req: dict) -> dict:
        ep = req["endpoint"]
        event = req.get("event", MembershipEvent.JOIN.value)
        if event == MembershipEvent.LEAVE.value:
            return self._reply(self.table.drop(tuple(ep["lid"]), "deregister"))
        self.table.put(ep, event)
        return self._reply(True)

    def _op_heartbeat(self, req: dict) -> dict:
        return self._reply(self.table.heartbeat(tuple(req["lid"])))

    def _op_report_failure(self, req: dict) -> dict:
        return self._reply(self.table.drop(tuple(req["lid"]), "reported"))

    def _op_lookup(self, req: dict) -> dict:
        ep = self.table.members.get(tuple(req["lid"]))
        return self._reply(True, endpoint=ep) if ep is not None else self._reply(False)

    def _op_list_stage(self, req: dict) -> dict:
        return self._reply(True, endpoints=[ep for _, ep in self.table.stage(req["model"], req["stage"])])

    def _op_assignment(self, req: dict) -> dict:
        found = self.table.stage(req.get("model"), req.get("target_stage"))
        if not found:
            return self._reply(False)
        key, ep = found[0]
        return self._reply(True, endpoint=ep["addresses"][0] if ep["addresses"] else "",
                           routing_key="-".join(str(x) for x in key))

    def _op_info(self, req: dict) -> dict:
        return self._reply(True, event_address=self.event_bind_addr, lease_s=self.lease_s)


def main() -> None:
    p = argparse.ArgumentParser(description="connex directory server")
    p.add_argument("--bind", default="127.0.0.1:5555")
    p.add_argument("--event-bind", default=None)
    p.add_argument("--lease", type=float, default=2.0)
    a = p.parse_args()
    logging.basicConfig(level=logging.INFO)
    try:
        DirectoryServer(a.bind, a.event_bind, a.lease).serve_forever()
    except KeyboardInterrupt:
        pass


if __name__ == "__main__":
    main()

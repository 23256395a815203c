"""In-memory directory service: ZeroMQ ROUTER for requests, PUB for events.

Speaks the :mod:`connex.directory` msgpack protocol (the reference's
``connex/directory_server.py:48-241``): a global epoch is bumped on every
membership change and returned in replies; every change is published as
``{"event", "endpoint", "epoch", "reason"}`` with reasons ``deregister``,
``reported`` or ``expired``.  Leases (``lease_s``) apply only to members that
have heartbeated at least once.

    python -m connex.directory_server --bind 127.0.0.1:5555
"""
from __future__ import annotations

import argparse
import logging
import threading
import time
from typing import Any, Optional

import msgpack
import zmq

from connex.directory import MembershipEvent

logger = logging.getLogger("connex.directory_server")


class DirectoryServer:
    def __init__(self, bind_addr: str = "127.0.0.1:5555", event_bind_addr: Optional[str] = None,
                 lease_s: float = 2.0):
        self.bind_addr = bind_addr
        host, port = bind_addr.rsplit(":", 1)
        self.event_bind_addr = event_bind_addr or f"{host}:{int(port) + 1}"
        self.lease_s = lease_s
        self.epoch = 0
        self._endpoints: dict = {}
        self._last_seen: dict = {}
        self._outbox: list = []
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._ready = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._bind_error: Optional[BaseException] = None

    # ------------------------------------------------------------ control
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
            return dict(self._endpoints)

    def serve_forever(self) -> None:
        ctx = zmq.Context.instance()
        sock, pub = ctx.socket(zmq.ROUTER), ctx.socket(zmq.PUB)
        for s in (sock, pub):
            s.setsockopt(zmq.LINGER, 0)
        try:
            sock.bind(f"tcp://{self.bind_addr}")
            pub.bind(f"tcp://{self.event_bind_addr}")
        except zmq.ZMQError as e:
            self._bind_error = e
            self._ready.set()
            sock.close()
            pub.close()
            return
        self._ready.set()
        tick_ms = int(1000 * min(0.05, self.lease_s / 4))
        try:
            while not self._stop.is_set():
                if sock.poll(tick_ms):
                    while True:  # drain the burst before publishing
                        try:
                            frames = sock.recv_multipart(zmq.NOBLOCK)
                        except zmq.Again:
                            break
                        try:
                            resp = self.handle(msgpack.unpackb(frames[-1], raw=False))
                        except Exception as e:
                            resp = {"status": "error", "error": str(e)}
                        sock.send_multipart([frames[0], msgpack.packb(resp, use_bin_type=True)])
                self._expire_leases()
                with self._lock:
                    out, self._outbox = self._outbox, []
                for ev in out:
                    pub.send(msgpack.packb(ev, use_bin_type=True))
        finally:
            sock.close()
            pub.close()

    # ----------------------------------------------------------- handlers
    def handle(self, req: dict) -> dict:
        kind = req.get("type")
        if kind == "register":
            return self._register(req)
        if kind == "heartbeat":
            return self._heartbeat(tuple(req["lid"]))
        if kind == "report_failure":
            with self._lock:
                ok = self._remove(tuple(req["lid"]), "reported")
                return {"status": "ok" if ok else "not_found", "epoch": self.epoch}
        if kind == "lookup":
            with self._lock:
                ep = self._endpoints.get(tuple(req["lid"]))
                if ep is None:
                    return {"status": "not_found", "epoch": self.epoch}
                return {"status": "ok", "endpoint": ep, "epoch": self.epoch}
        if kind == "list_stage":
            with self._lock:
                eps = [ep for lid, ep in sorted(self._endpoints.items())
                       if lid[0] == req["model"] and lid[1] == req["stage"]]
                return {"status": "ok", "endpoints": eps, "epoch": self.epoch}
        if kind == "request_assignment":
            return self._assignment(req)
        if kind == "info":
            return {"status": "ok", "event_address": self.event_bind_addr, "lease_s": self.lease_s,
                    "epoch": self.epoch}
        return {"status": "error", "error": f"unknown request type {kind!r}"}

    def _publish(self, event: str, ep: dict, reason: str) -> None:
        self.epoch += 1
        self._outbox.append({"event": event, "endpoint": ep, "epoch": self.epoch, "reason": reason})

    def _remove(self, lid: tuple, reason: str) -> bool:  # lock held
        ep = self._endpoints.pop(lid, None)
        self._last_seen.pop(lid, None)
        if ep is None:
            return False
        self._publish(MembershipEvent.LEAVE.value, ep, reason)
        logger.info("LEAVE %s (%s, epoch %d)", lid, reason, self.epoch)
        return True

    def _register(self, req: dict) -> dict:
        ep = req["endpoint"]
        lid = tuple(ep["lid"])
        event = req.get("event", MembershipEvent.JOIN.value)
        with self._lock:
            if event == MembershipEvent.LEAVE.value:
                ok = self._remove(lid, "deregister")
                return {"status": "ok" if ok else "not_found", "epoch": self.epoch}
            self._endpoints[lid] = ep
            if lid in self._last_seen:
                self._last_seen[lid] = time.monotonic()
            self._publish(event, ep, "")
            return {"status": "ok", "epoch": self.epoch}

    def _heartbeat(self, lid: tuple) -> dict:
        with self._lock:
            if lid not in self._endpoints:
                return {"status": "not_found", "epoch": self.epoch}
            self._last_seen[lid] = time.monotonic()
            return {"status": "ok", "epoch": self.epoch}

    def _expire_leases(self) -> None:
        now = time.monotonic()
        with self._lock:
            for lid in [l for l, t in self._last_seen.items() if now - t > self.lease_s]:
                self._remove(lid, "expired")

    def _assignment(self, req: dict) -> dict:
        model, stage = req.get("model"), req.get("target_stage")
        with self._lock:
            cands = sorted(l for l in self._endpoints if l[0] == model and l[1] == stage)
            if not cands:
                return {"status": "not_found", "epoch": self.epoch}
            ep = self._endpoints[cands[0]]
            return {"status": "ok", "endpoint": ep["addresses"][0] if ep["addresses"] else "",
                    "routing_key": "-".join(str(x) for x in cands[0]), "epoch": self.epoch}


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

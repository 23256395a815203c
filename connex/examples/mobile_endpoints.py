"""Mobility run: one sender, one downstream logical group with replicas that
fail, rejoin, migrate and leave while steps are in flight.

    python -m connex.examples.mobile_endpoints --steps 1000

Workload (CPU only): a directory server in-process, the sender and every
replica talk ZeroMQ/TCP on 127.0.0.1.  Each step carries a 64-byte payload
drawn from ``seed``; the sender uses :class:`connex.elastic.ElasticPeerSet`
to pick a live replica of stage 1 and waits for that replica's ack before
the next step (one step in flight, so delivery order is the step order).
A step whose ack does not arrive is re-sent under the same correlation id
to another replica after ``mark_failed``; replicas drop correlation ids they
already processed (receiver dedupe).  Scripted events (defaults from the
reference's mobility example, ``examples/mobile_endpoints.py``):

* ``fail_at``:    the sender marks replica 1 failed (reported to the directory)
* ``rejoin_at``:  replica 1 registers again (same identity, same address)
* ``migrate_at``: replica 0 moves to a new address under the same identity
* ``leave_at``:   replica 0 deregisters

The report lists every delivery so a checker can verify that each step was
delivered exactly once, in order, to a replica that was live at the time.
"""
from __future__ import annotations

import argparse
import json
import random
import struct
import threading
import time
from typing import Dict, List, Optional

import zmq

from connex.directory import DirectoryClient, MembershipEvent
from connex.directory_server import DirectoryServer
from connex.elastic import ElasticPeerSet, ZmqTransport

MODEL = "mobility"
HDR = struct.Struct("!QQ")  # corr, sender ack port


def _free_port() -> int:
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class Replica:
    """A stage-1 replica: PULL socket(s), receiver dedupe, acks to the sender."""

    def __init__(self, directory_addr: str, replica_idx: int, log: List[dict], log_lock: threading.Lock):
        self.idx = replica_idx
        self.log, self.log_lock = log, log_lock
        self.ctx = zmq.Context.instance()
        self.client = DirectoryClient(directory_addr, MODEL, 1, replica_idx=replica_idx)
        self.client.start()
        self.seen: set = set()
        self.live = False
        self._socks: List[zmq.Socket] = []
        self._acks: Dict[int, zmq.Socket] = {}
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self.address = self._listen()
        self._thread = threading.Thread(target=self._loop, daemon=True, name=f"replica-{replica_idx}")
        self._thread.start()

    def _listen(self) -> str:
        s = self.ctx.socket(zmq.PULL)
        s.setsockopt(zmq.LINGER, 0)
        port = s.bind_to_random_port("tcp://127.0.0.1")
        with self._lock:
            self._socks.append(s)
        return f"127.0.0.1:{port}"

    def join(self) -> None:
        self.live = True
        assert self.client.register([self.address])

    def migrate(self) -> str:
        """Listen on a new address and move the same LID there; the old
        socket keeps draining until ``close_old``."""
        self.address = self._listen()
        assert self.client.notify_migration([self.address], self.client.get_current_epoch() + 1)
        return self.address

    def close_old(self) -> None:
        with self._lock:
            old, self._socks = self._socks[:-1], self._socks[-1:]
        time.sleep(0.05)  # let the receive loop switch to the new socket set first
        for s in old:
            s.close(0)

    def leave(self) -> None:
        self.live = False
        self.client.deregister()

    def _ack(self, port: int, corr: int) -> None:
        s = self._acks.get(port)
        if s is None:
            s = self.ctx.socket(zmq.PUSH)
            s.setsockopt(zmq.LINGER, 0)
            s.connect(f"tcp://127.0.0.1:{port}")
            self._acks[port] = s
        s.send(HDR.pack(corr, self.idx))

    def _loop(self) -> None:
        poller_socks: List[zmq.Socket] = []
        while not self._stop.is_set():
            with self._lock:
                socks = list(self._socks)
            if socks != poller_socks:
                poller = zmq.Poller()
                for s in socks:
                    poller.register(s, zmq.POLLIN)
                poller_socks = socks
            try:
                ready = poller.poll(20)
            except zmq.ZMQError:  # a socket was closed by close_old() meanwhile
                poller_socks = []
                continue
            for s, _ in ready:
                try:
                    msg = s.recv(zmq.NOBLOCK)
                except zmq.ZMQError:
                    continue
                corr, port = HDR.unpack_from(msg)
                payload = msg[HDR.size:]
                if corr not in self.seen:  # receiver dedupe (idempotent re-send)
                    self.seen.add(corr)
                    with self.log_lock:
                        self.log.append({"corr": corr, "replica": self.idx, "payload": payload.hex(),
                                         "live": self.live, "t": time.monotonic()})
                self._ack(port, corr)

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(2)
        for s in self._socks + list(self._acks.values()):
            s.close(0)
        self.client.stop()


def run(steps: int = 1000, seed: int = 0, payload_bytes: int = 64, fail_at: int = 200, rejoin_at: int = 400,
        migrate_at: int = 600, leave_at: int = 800, ack_timeout_s: float = 1.0) -> dict:
    dport = _free_port()
    server = DirectoryServer(f"127.0.0.1:{dport}", lease_s=2.0)
    server.start()
    log: List[dict] = []
    lock = threading.Lock()
    replicas = [Replica(server.bind_addr, r, log, lock) for r in range(2)]
    for r in replicas:
        r.join()
    sender_dir = DirectoryClient(server.bind_addr, MODEL, 0)
    sender_dir.start()
    transport = ZmqTransport()
    peers = ElasticPeerSet(sender_dir, transport, stage_idx=1, drain_grace_s=0.5)
    peers.start()
    if not peers.wait_ready(2, timeout=10):
        raise RuntimeError("replicas did not become routable")
    ack = zmq.Context.instance().socket(zmq.PULL)
    ack.setsockopt(zmq.LINGER, 0)
    ack_port = ack.bind_to_random_port("tcp://127.0.0.1")
    rng = random.Random(seed)
    sent: List[dict] = []
    events: List[dict] = []
    resends = 0
    t0 = time.monotonic()
    for i in range(steps):
        if i == fail_at:
            peers.mark_failed((MODEL, 1, 0, 1))
            replicas[1].live = False
            events.append({"step": i, "event": "fail", "replica": 1})
        elif i == rejoin_at:
            replicas[1].join()
            peers.wait_ready(2, timeout=10)
            events.append({"step": i, "event": "rejoin", "replica": 1})
        elif i == migrate_at:
            addr = replicas[0].migrate()
            # wait until the sender routes replica 0 to its new address
            deadline = time.monotonic() + 10
            while time.monotonic() < deadline and peers.address((MODEL, 1, 0, 0)) != addr:
                time.sleep(0.005)
            replicas[0].close_old()
            events.append({"step": i, "event": "migrate", "replica": 0, "address": addr})
        elif i == leave_at:
            replicas[0].leave()
            deadline = time.monotonic() + 10
            while time.monotonic() < deadline and (MODEL, 1, 0, 0) in peers.peers():
                time.sleep(0.005)
            events.append({"step": i, "event": "leave", "replica": 0})
        payload = bytes(rng.getrandbits(8) for _ in range(payload_bytes))
        corr = i
        msg = HDR.pack(corr, ack_port) + payload
        sent.append({"corr": corr, "payload": payload.hex()})
        while True:
            lid = peers.pick()
            if lid is None:
                peers.wait_ready(1, timeout=5)
                continue
            try:
                peers.send(lid, msg)
            except Exception:
                resends += 1
                continue
            if ack.poll(int(ack_timeout_s * 1000)):
                got, _rep = HDR.unpack(ack.recv())
                if got == corr:
                    break
            peers.mark_failed(lid)
            resends += 1
    elapsed = time.monotonic() - t0
    ack.close(0)
    peers.stop()
    transport.stop_sync()
    sender_dir.stop()
    for r in replicas:
        r.stop()
    server.stop()
    return {"steps": steps, "sent": sent, "deliveries": log, "events": events, "resends": resends,
            "elapsed_s": elapsed, "peer_stats": peers.stats}


def check(report: dict) -> dict:
    """Exactly once, in order, each to a live replica, payloads intact."""
    dl = sorted(report["deliveries"], key=lambda d: d["t"])
    corrs = [d["corr"] for d in dl]
    ok_once = sorted(corrs) == list(range(report["steps"])) and len(set(corrs)) == len(corrs)
    ok_order = corrs == sorted(corrs)
    ok_live = all(d["live"] for d in dl)
    sent = {s["corr"]: s["payload"] for s in report["sent"]}
    ok_payload = all(sent.get(d["corr"]) == d["payload"] for d in dl)
    by_replica = {}
    for d in dl:
        by_replica[d["replica"]] = by_replica.get(d["replica"], 0) + 1
    return {"exactly_once": ok_once, "in_order": ok_order, "live_only": ok_live, "payload_ok": ok_payload,
            "per_replica": by_replica, "resends": report["resends"], "elapsed_s": report["elapsed_s"]}


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args()
    print(json.dumps(check(run(a.steps, a.seed))))


if __name__ == "__main__":
    main()

"""Control-plane load test of the directory (``connex-directory``): register
``--endpoints`` endpoints, then for ``--duration-s`` seconds ``--updaters``
processes re-register (MIGRATE) random endpoints as fast as the server
answers, while one process times lookups (request -> answer) and one
subscriber times update -> event delivery (each update carries its send
time in its address).  Reports update throughput, lookup and notification
latency percentiles and the server's CPU seconds.  CPU only.

    python -m connex_b200.bench.control_plane_bench --endpoints 2000 --updaters 4 --duration-s 10

Reference counterpart: ``benchmarks/control_plane_bench.py`` (same
workload shape against its directory server).
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import random
import time

import zmq

from connex.directory import MembershipEvent, _pack, _unpack

MODEL = "cpbench"


def _pct(xs, q):
    xs = sorted(xs)
    return round(xs[min(len(xs) - 1, int(q * len(xs)))] * 1e3, 3) if xs else None


def _ep(i: int, addr: str) -> dict:
    return {"lid": [MODEL, 1, 0, i], "addresses": [addr], "transport_caps": ["zeromq"], "epoch": 0, "state": "active"}


class _Conn:
    def __init__(self, addr: str):
        self.s = zmq.Context.instance().socket(zmq.DEALER)
        self.s.setsockopt(zmq.LINGER, 0)
        self.s.connect(f"tcp://{addr}")

    def call(self, msg: dict, timeout_ms: int = 5000) -> dict:
        self.s.send(_pack(msg))
        if not self.s.poll(timeout_ms):
            raise TimeoutError(msg.get("type"))
        return _unpack(self.s.recv())


def _updater(addr, n, duration, seed, q, go):
    c, rng = _Conn(addr), random.Random(seed)
    go.wait()
    done, end = 0, time.monotonic() + duration
    while time.monotonic() < end:
        i = rng.randrange(n)
        c.call({"type": "register", "event": MembershipEvent.MIGRATE.value,
                "endpoint": _ep(i, f"tcp://10.0.0.1:{20000 + i}#t={time.time():.6f}")})
        done += 1
    q.put(("updates", done))


def _looker(addr, n, duration, seed, q, go):
    c, rng, lat = _Conn(addr), random.Random(seed), []
    go.wait()
    end = time.monotonic() + duration
    while time.monotonic() < end:
        t0 = time.perf_counter()
        r = c.call({"type": "lookup", "lid": [MODEL, 1, 0, rng.randrange(n)]})
        lat.append(time.perf_counter() - t0)
        assert r.get("status") == "ok"
    q.put(("lookups", lat))


def _subscriber(event_addr, duration, q, go, ready):
    s = zmq.Context.instance().socket(zmq.SUB)
    s.setsockopt(zmq.SUBSCRIBE, b"")
    s.setsockopt(zmq.LINGER, 0)
    s.connect(f"tcp://{event_addr}")
    time.sleep(0.3)                          # the subscription reaches the publisher
    ready.set()
    go.wait()
    delays, end = [], time.monotonic() + duration + 1.0
    while time.monotonic() < end:
        if not s.poll(100):
            continue
        ev = _unpack(s.recv())
        for a in ev.get("endpoint", {}).get("addresses", []):
            if "#t=" in a:
                delays.append(time.time() - float(a.split("#t=", 1)[1]))
    q.put(("events", delays))


def _cpu_s(pid: int) -> float:
    try:
        with open(f"/proc/{pid}/stat") as f:
            parts = f.read().rsplit(")", 1)[1].split()
        return (int(parts[11]) + int(parts[12])) / os.sysconf("SC_CLK_TCK")
    except OSError:
        return float("nan")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--endpoints", type=int, default=2000)
    ap.add_argument("--updaters", type=int, default=4)
    ap.add_argument("--duration-s", type=float, default=10.0)
    ap.add_argument("--port", type=int, default=0)
    a = ap.parse_args(argv)
    print(json.dumps(bench(a.endpoints, a.updaters, a.duration_s, a.port)))
    return 0


def bench(endpoints: int, updaters: int, duration_s: float, port: int = 0) -> dict:
    import socket
    import subprocess
    import sys
    if not port:
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
    addr, ev_addr = f"127.0.0.1:{port}", f"127.0.0.1:{port + 1}"
    server = subprocess.Popen([sys.executable, "-m", "connex.directory_server", "--bind", addr, "--event-bind",
                               ev_addr, "--lease", "3600"], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    try:
        c = _Conn(addr)
        t_end = time.monotonic() + 30
        while True:
            try:
                c.call({"type": "info"}, 500)
                break
            except TimeoutError:
                if time.monotonic() > t_end:
                    raise
        t0 = time.perf_counter()
        for i in range(endpoints):
            assert c.call({"type": "register", "event": MembershipEvent.JOIN.value,
                           "endpoint": _ep(i, f"tcp://10.0.0.1:{20000 + i}")})["status"] == "ok"
        reg_s = time.perf_counter() - t0
        ctx = mp.get_context("fork")
        q, go, ready = ctx.Queue(), ctx.Event(), ctx.Event()
        procs = [ctx.Process(target=_subscriber, args=(ev_addr, duration_s, q, go, ready))]
        procs += [ctx.Process(target=_updater, args=(addr, endpoints, duration_s, k, q, go)) for k in range(updaters)]
        procs += [ctx.Process(target=_looker, args=(addr, endpoints, duration_s, 99, q, go))]
        for p in procs:
            p.start()
        ready.wait(10)
        cpu0 = _cpu_s(server.pid)
        go.set()
        got = [q.get(timeout=duration_s + 60) for _ in procs]
        cpu1 = _cpu_s(server.pid)
        for p in procs:
            p.join(10)
        updates = sum(v for k, v in got if k == "updates")
        lookups = [x for k, v in got if k == "lookups" for x in v]
        events = [x for k, v in got if k == "events" for x in v]
        return {"endpoints": endpoints, "updaters": updaters, "duration_s": duration_s,
                "register_per_s": round(endpoints / reg_s, 1), "updates_per_s": round(updates / duration_s, 1),
                "lookups": len(lookups), "lookup_p50_ms": _pct(lookups, 0.5), "lookup_p99_ms": _pct(lookups, 0.99),
                "events": len(events), "notify_p50_ms": _pct(events, 0.5), "notify_p99_ms": _pct(events, 0.99),
                "server_cpu_s": round(cpu1 - cpu0, 2)}
    finally:
        server.terminate()
        server.wait(10)


if __name__ == "__main__":
    raise SystemExit(main())

"""Pipeline failover details over real sockets on CPU: probing (alive, dead,
unknown), a missed lease that only makes the downstream suspect (kept while
it accepts connects, failed over at once when its port refuses), events about
unrelated replicas, K steps in flight failing over together and re-sent under
their own ids, waiters woken by a failover, replies matched by id out of
order and across concurrent waiters, and the adaptive step timeout."""
import socket
import threading
import time

import pytest
import torch

from connex.front_router import EventType
from connex.pp.endpoint import PipelineEndpoint, probe_tcp
from connex.pp.link import Stage0Link, StageWorker
from connex.pp.routing import StaticMembership
from tests.helpers import free_port, wait_until


class Hooks:
    def kv_held(self, rid):
        return 0

    def release(self, rids):
        pass

    def reprefill(self, rids):
        pass

    def abort(self, rids):
        pass


def _serve(ep, add, stop, delay=0.0):
    w = StageWorker(ep, Hooks(), lambda td, missing: (time.sleep(delay), {"x": td["x"] + add})[1])

    def loop():
        while not stop.is_set():
            try:
                w.serve_one()
            except Exception:
                if stop.is_set():                # the endpoint was closed under a slow step
                    return
                raise
    t = threading.Thread(target=loop, daemon=True)
    t.start()
    return t


def _two_replicas(k=1, timeout=1.0):
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, 0, membership=mem, k=k, recv_timeout_s=timeout)
    a = PipelineEndpoint("m", 1, 2, 0, membership=mem, k=k, recv_timeout_s=timeout)
    b = PipelineEndpoint("m", 1, 2, 1, membership=mem, k=k, recv_timeout_s=timeout)
    for e in (s0, a, b):
        mem.add(e.stage_idx, e.replica_idx, e.address)
    return mem, s0, a, b


def test_probe_alive_dead_unknown():
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    try:
        assert probe_tcp(f"tcp://127.0.0.1:{srv.getsockname()[1]}#x") is True
        assert probe_tcp(f"tcp://127.0.0.1:{free_port()}") is False
        assert probe_tcp("inproc://nothing") is None and probe_tcp(None) is None
    finally:
        srv.close()


def test_unhealthy_but_alive_downstream_is_kept():
    mem, s0, a, b = _two_replicas()
    stop = threading.Event()
    _serve(a, 10, stop)
    _serve(b, 20, stop)
    try:
        link = Stage0Link(s0, Hooks(), recv_timeout_s=1.0)
        first = link.step({"x": torch.zeros(1)})["x"].item()
        cur = s0.current
        mem.emit(EventType.ENDPOINT_UNHEALTHY, 1, cur)               # late heartbeat, process alive
        assert wait_until(lambda: s0.stats["suspect_alive"] == 1, 3)
        assert s0.current == cur and s0.stats["failovers"] == 0
        assert link.step({"x": torch.zeros(1)})["x"].item() == first
        mem.emit(EventType.ENDPOINT_REGISTERED, 1, cur)
        assert (1, cur) not in s0.suspect
    finally:
        stop.set()
        for e in (s0, a, b):
            e.close()


def test_unhealthy_and_refusing_downstream_fails_over_without_waiting_for_the_lease():
    mem, s0, a, b = _two_replicas(timeout=5.0)
    stops = {a: threading.Event(), b: threading.Event()}
    _serve(a, 10, stops[a])
    _serve(b, 20, stops[b])
    try:
        link = Stage0Link(s0, Hooks(), recv_timeout_s=5.0)
        link.step({"x": torch.zeros(1)})
        victim = a if s0.current == a.replica_idx else b
        stops[victim].set()
        victim.close()                                                 # port closed: connects refused
        mem.emit(EventType.ENDPOINT_UNHEALTHY, 1, victim.replica_idx)
        assert wait_until(lambda: s0.stats["failovers"] == 1, 3)
        t0 = time.monotonic()
        out = link.step({"x": torch.zeros(1)})["x"].item()
        assert out == (20 if victim is a else 10) and time.monotonic() - t0 < 2.0
    finally:
        for e in stops.values():
            e.set()
        for e in (s0, a, b):
            if e is not victim:
                e.close()


def test_events_about_other_replicas_change_nothing():
    mem, s0, a, b = _two_replicas()
    stop = threading.Event()
    _serve(a, 10, stop)
    _serve(b, 20, stop)
    try:
        link = Stage0Link(s0, Hooks(), recv_timeout_s=1.0)
        link.step({"x": torch.zeros(1)})
        other = 1 - s0.current
        mem.emit(EventType.ENDPOINT_UNHEALTHY, 1, other)
        mem.emit(EventType.ENDPOINT_UNHEALTHY, 2, 0)                   # a stage we do not send to
        time.sleep(0.2)
        assert not s0.suspect and s0.stats["failovers"] == 0 and s0.stats["suspect_alive"] == 0
    finally:
        stop.set()
        for e in (s0, a, b):
            e.close()


def test_k_steps_in_flight_fail_over_together_and_keep_their_ids():
    mem, s0, a, b = _two_replicas(k=3, timeout=3.0)
    stops = {a: threading.Event(), b: threading.Event()}
    _serve(b, 20, stops[b])                                            # only b answers
    _serve(a, 10, stops[a], delay=4.0)                                 # a takes steps and does not answer in time
    try:
        link = Stage0Link(s0, Hooks(), recv_timeout_s=3.0)
        s0.set_downstream(a.address, a.replica_idx)
        s0.membership = None                                           # pin to a first
        corrs = [link.submit({"x": torch.full((1,), float(i))}) for i in range(3)]
        s0.membership = mem
        assert s0.on_peer_dead(1, a.replica_idx, "killed")
        t0 = time.monotonic()
        outs = [link.wait(c)["x"].item() for c in corrs]
        assert outs == [20.0, 21.0, 22.0] and time.monotonic() - t0 < 2.5
        assert link.stats["retries"] >= 3                              # every in-flight step was re-sent
    finally:
        for e in stops.values():
            e.set()
        for e in (s0, a, b):
            e.close()


def test_a_waiting_receive_is_woken_by_the_failover():
    mem, s0, a, b = _two_replicas(timeout=30.0)
    try:
        corr = s0.new_step_id()
        s0.send_step({"x": torch.zeros(1)}, corr)                       # nobody serves: no reply
        got = {}

        def wait():
            t0 = time.monotonic()
            got["r"] = s0.recv_step(corr, 30.0)
            got["dt"] = time.monotonic() - t0
        t = threading.Thread(target=wait)
        t.start()
        time.sleep(0.2)
        s0.on_peer_dead(1, s0.current, "killed")
        t.join(5)
        assert got["r"] is None and got["dt"] < 2.0 and s0.step_stale(corr)
    finally:
        for e in (s0, a, b):
            e.close()


def test_out_of_order_replies_and_concurrent_waiters():
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, membership=mem, k=4, recv_timeout_s=5.0)
    s1 = PipelineEndpoint("m", 1, 2, membership=mem, k=4, recv_timeout_s=5.0)
    mem.add(0, 0, s0.address)
    mem.add(1, 0, s1.address)
    try:
        corrs = [s0.new_step_id() for _ in range(4)]
        for i, c in enumerate(corrs):
            s0.send_step({"x": torch.full((1,), float(i))}, c)
        got = [s1.recv_forward(2.0) for _ in range(4)]
        results = {}

        def wait(c):
            results[c] = s0.recv_step(c, 5.0)
        ts = [threading.Thread(target=wait, args=(c,)) for c in corrs]
        for t in ts:
            t.start()
        for td, ctx in reversed(got):                                    # answered last-first
            s1.send_reply({"x": td["x"] * 10}, ctx)
        for t in ts:
            t.join(5)
        assert [results[c]["x"].item() for c in corrs] == [0.0, 10.0, 20.0, 30.0]
    finally:
        s0.close()
        s1.close()


def test_step_timeout_follows_the_slowest_measured_step():
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, membership=mem, recv_timeout_s=0.5)
    s1 = PipelineEndpoint("m", 1, 2, membership=mem, recv_timeout_s=0.5)
    mem.add(0, 0, s0.address)
    mem.add(1, 0, s1.address)
    stop = threading.Event()
    _serve(s1, 1, stop, delay=0.3)
    try:
        assert s0._recv_timeout_s() == pytest.approx(0.5)
        link = Stage0Link(s0, Hooks(), recv_timeout_s=None)
        link.step({"x": torch.zeros(1)})
        assert s0.slowest_step_s >= 0.3 and s0._recv_timeout_s() >= 0.9   # 3x the slowest step
    finally:
        stop.set()
        s0.close()
        s1.close()

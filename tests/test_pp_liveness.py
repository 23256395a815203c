"""The pipeline's failure tiers on CPU, over real sockets: transport peer-death
events (a stage process SIGKILLed: the native engine reports it, stage 0 re-
routes without any lease or probe), the stage-0 watchdog (adaptive step
timeout, ping of the route, pick-stuck for a replica that answers pings but
no longer answers steps), DYING, ownership with BUSY and takeover, READY from
a restarted replica via its head-state file, and the false-failure check for
a replica that rejoined and still answers."""
import multiprocessing as mp
import os
import signal
import threading
import time

import pytest
import torch

from connex.pp.endpoint import PipelineEndpoint
from connex.pp.link import Stage0Link, StageWorker
from connex.pp.liveness import ChainWatchdog, HeadState, Hop, StageResponder, pick_stuck
from connex.pp.routing import StaticMembership
from tests.helpers import wait_until


class Hooks:
    def kv_held(self, rid):
        return 0

    def release(self, rids):
        pass

    def reprefill(self, rids):
        pass

    def abort(self, rids):
        pass


def _serve(ep, add, stop, delay=0.0, gate=None):
    """A stage worker thread: x -> x + add.  ``gate`` (an Event) holds its
    compute while cleared: the replica then still answers pings but no steps."""
    def compute(td, missing):
        while gate is not None and not gate.is_set() and not stop.is_set():
            time.sleep(0.01)
        time.sleep(delay)
        return {"x": td["x"] + add}
    w = StageWorker(ep, Hooks(), compute)

    def loop():
        while not stop.is_set():
            try:
                w.serve_one()
            except Exception:
                if stop.is_set():
                    return
                raise
    t = threading.Thread(target=loop, daemon=True)
    t.start()
    return t


def _chain(tmp_path, timeout=30.0):
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, 0, membership=mem, recv_timeout_s=timeout)
    a = PipelineEndpoint("m", 1, 2, 0, membership=mem, recv_timeout_s=timeout)
    b = PipelineEndpoint("m", 1, 2, 1, membership=mem, recv_timeout_s=timeout)
    for e in (s0, a, b):
        mem.add(e.stage_idx, e.replica_idx, e.address)
    ra, rb = StageResponder(a, state_dir=str(tmp_path)), StageResponder(b, state_dir=str(tmp_path))
    return mem, s0, a, b, ra, rb


def _close(*eps):
    for e in eps:
        e.close()


def test_pick_stuck_rules():
    route = [Hop(1, 0, "a", pong=5.0, done_seq=10), Hop(2, 0, "b", pong=5.0, done_seq=8)]
    assert pick_stuck(route, [], 4.0) == (None, "")
    assert pick_stuck(route, [9], 4.0)[0].address == "b"          # stage 2 has not finished step 9
    route[1].pong = 3.0
    hop, why = pick_stuck(route, [9], 4.0)
    assert hop.address == "b" and "no pong" in why
    route[1].pong, route[1].done_seq = 5.0, 20
    assert pick_stuck(route, [9], 4.0)[0].address == "b"          # everyone is ahead: the last one


def test_adaptive_step_timeout_follows_like_sized_steps():
    class Ep:
        control_handlers, route_listeners, failure_veto = [], [], None

    class Link:
        step_listeners = []
    wd = ChainWatchdog(Ep(), Link(), step_timeout=60.0, min_timeout=2.0, factor=20.0, min_samples=4)
    assert wd.current_step_timeout(1) == 60.0                      # too few samples: the backstop
    for _ in range(4):
        wd.record(0.01, 1)                                         # small decode steps
    wd.record(0.5, 4096)                                           # one long prefill
    assert wd.current_step_timeout(1) == pytest.approx(10.0)       # 20 x 0.5 s
    assert wd.current_step_timeout(4096) == pytest.approx(10.0)
    assert wd.current_step_timeout(8192) == 60.0                   # larger than any measured step
    wd2 = ChainWatchdog(Ep(), Link(), min_samples=4, min_timeout=2.0)
    for _ in range(4):
        wd2.record(0.001, 1)
    assert wd2.current_step_timeout(1) == 2.0                      # clamped to the minimum


def test_watchdog_fails_over_a_replica_that_answers_pings_but_not_steps(tmp_path):
    mem, s0, a, b, ra, rb = _chain(tmp_path)
    stop, gate = threading.Event(), threading.Event()
    gate.set()
    _serve(a, 10, stop, gate=gate)
    _serve(b, 20, stop)
    link = Stage0Link(s0, Hooks(), recv_timeout_s=30.0)
    wd = ChainWatchdog(s0, link, step_timeout=1.0, ping_wait_s=0.3, period_s=0.1)
    try:
        assert link.step({"x": torch.zeros(1)})["x"].item() == 10          # routed to replica a
        assert wait_until(lambda: ra.owner == s0.address, 3)                # HELLO -> owner
        gate.clear()                                                        # a hangs (its I/O still answers)
        wd.start()
        t0 = time.monotonic()
        out = link.step({"x": torch.zeros(1)})["x"].item()
        assert out == 20 and time.monotonic() - t0 < 5.0                    # re-sent to b after the timeout
        assert wd.events and wd.events[-1]["replica"] == 0 and "answers but is stuck" in wd.events[-1]["reason"]
        assert wd.stats["late_rounds"] >= 1
    finally:
        stop.set()
        gate.set()
        wd.stop()
        _close(s0, a, b)


def test_dying_replica_is_failed_over_at_once(tmp_path):
    mem, s0, a, b, ra, rb = _chain(tmp_path)
    stop = threading.Event()
    _serve(a, 10, stop)
    _serve(b, 20, stop)
    link = Stage0Link(s0, Hooks(), recv_timeout_s=30.0)
    wd = ChainWatchdog(s0, link)
    try:
        assert link.step({"x": torch.zeros(1)})["x"].item() == 10
        assert wait_until(lambda: ra.owner == s0.address, 3)
        ra.dying("SIGTERM")
        assert wait_until(lambda: s0.current == 1 or (1, 0) in s0.deregistered, 3)
        assert wd.stats["dying"] == 1
        assert link.step({"x": torch.zeros(1)})["x"].item() == 20
    finally:
        stop.set()
        _close(s0, a, b)


def test_owned_replica_answers_busy_until_its_owner_goes_silent(tmp_path):
    mem = StaticMembership(0, 0)
    h1 = PipelineEndpoint("m", 0, 2, 0, membership=mem, recv_timeout_s=5.0)
    h2 = PipelineEndpoint("m", 0, 2, 1, membership=mem, recv_timeout_s=5.0)
    a = PipelineEndpoint("m", 1, 2, 0, membership=mem, recv_timeout_s=5.0)
    ra = StageResponder(a, state_dir=str(tmp_path), takeover_s=0.5)
    got = {"h1": [], "h2": []}
    h1.control_handlers.append(lambda m: got["h1"].append(m["kind"]))
    h2.control_handlers.append(lambda m: got["h2"].append(m["kind"]))
    try:
        h1.send_control(a.address, {"kind": "HELLO"})
        assert wait_until(lambda: "HELLO_OK" in got["h1"], 3)
        h2.send_control(a.address, {"kind": "HELLO"})
        assert wait_until(lambda: "BUSY" in got["h2"], 3) and ra.owner == h1.address
        time.sleep(0.7)                                             # h1 silent past the takeover time
        h2.send_control(a.address, {"kind": "HELLO"})
        assert wait_until(lambda: "HELLO_OK" in got["h2"], 3) and ra.owner == h2.address
        assert ra.stats["takeovers"] == 1
        # both heads are remembered for the announce after a restart
        assert HeadState(ra.heads.path).heads == [h1.address, h2.address]
    finally:
        _close(h1, h2, a)


def test_restarted_replica_announces_ready_and_rejoins(tmp_path):
    mem, s0, a, b, ra, rb = _chain(tmp_path)
    stop = threading.Event()
    _serve(a, 10, stop)
    link = Stage0Link(s0, Hooks(), recv_timeout_s=30.0)
    wd = ChainWatchdog(s0, link)
    try:
        assert link.step({"x": torch.zeros(1)})["x"].item() == 10
        assert wait_until(lambda: ra.owner == s0.address, 3)
        s0.on_peer_dead(1, 0, "test")                               # a was declared dead meanwhile
        assert (1, 0) in s0.deregistered
        # a restarted replica under the same identity finds its head in the state file
        a2 = PipelineEndpoint("m", 1, 2, 0, membership=mem, recv_timeout_s=5.0)
        ra2 = StageResponder(a2, state_dir=str(tmp_path))
        assert ra2.announce() == 1
        assert wait_until(lambda: wd.stats["ready"] == 1 and (1, 0) not in s0.deregistered, 3)
        assert wait_until(lambda: ra2.owner == s0.address, 3)       # stage 0 answered READY with HELLO
        a2.close()
    finally:
        stop.set()
        _close(s0, a, b)


def test_failure_report_about_a_rejoined_replica_that_answers_is_ignored(tmp_path):
    mem, s0, a, b, ra, rb = _chain(tmp_path)
    stop = threading.Event()
    _serve(a, 10, stop)
    link = Stage0Link(s0, Hooks(), recv_timeout_s=30.0)
    wd = ChainWatchdog(s0, link)
    try:
        assert link.step({"x": torch.zeros(1)})["x"].item() == 10
        assert wait_until(lambda: wd.hops.get((1, 0)) is not None and wd.hops[(1, 0)].alive_since > 0, 3)
        assert wd.vetoes(1, 0) is True and wd.stats["false_failures"] == 1
        a.close()                                                   # now it is really gone
        assert wd.vetoes(1, 0) is False
    finally:
        stop.set()
        _close(s0, b)


# ------------------------------------------------- transport tier, real processes
def _stage_process(replica, q, stop_path):
    """A stage-1 replica process: endpoint + native engine + worker."""
    from connex_b200.engine import Engine
    mem = StaticMembership(1, replica)
    ep = PipelineEndpoint("m", 1, 2, replica, membership=mem, recv_timeout_s=30.0)
    eng = Engine("m", 1, 0, replica, listen_ip="127.0.0.1")
    q.put((replica, ep.address, eng.local_url, os.getpid()))
    stop = threading.Event()
    _serve(ep, 10 * (replica + 1), stop, delay=0.3 if replica == 0 else 0.0)
    while not os.path.exists(stop_path):
        time.sleep(0.05)
    stop.set()
    ep.close()
    eng.close()


def test_sigkilled_stage_is_rerouted_on_the_transport_event(tmp_path):
    pytest.importorskip("connex_b200._cxengine")
    from connex_b200.engine import Engine
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    stop_path = str(tmp_path / "stop")
    procs = {r: ctx.Process(target=_stage_process, args=(r, q, stop_path), daemon=True) for r in (0, 1)}
    for p in procs.values():
        p.start()
    info = {}
    for _ in range(2):
        r, addr, url, pid = q.get(timeout=120)
        info[r] = (addr, url, pid)
    mem = StaticMembership(0, 0)
    for r, (addr, _, _) in info.items():
        mem.add(1, r, addr)
    s0 = PipelineEndpoint("m", 0, 2, 0, membership=mem, recv_timeout_s=30.0)   # no timeout path in play
    eng = Engine("m", 0, 0, 0, listen_ip="127.0.0.1")
    s0.watch_peers(eng, {(1, r): url for r, (_, url, _) in info.items()})
    link = Stage0Link(s0, Hooks(), recv_timeout_s=30.0)
    try:
        assert wait_until(lambda: len(s0._transport_up) == 2, 10)
        assert link.step({"x": torch.zeros(1)})["x"].item() == 10                # replica 0
        corr = link.submit({"x": torch.zeros(1)})                              # in flight on replica 0 (0.3 s)
        time.sleep(0.05)
        t_kill = time.monotonic()
        os.kill(info[0][2], signal.SIGKILL)
        out = link.wait(corr)["x"].item()
        t_done = time.monotonic()
        assert out == 20                                                       # re-sent to replica 1
        fo = s0.last_transport_failover
        assert fo is not None and fo["peer"] == (1, 0)
        assert fo["failover_t"] - fo["event_t"] < 0.1                          # event -> re-route
        assert fo["failover_t"] - t_kill < 1.0 and t_done - t_kill < 2.0        # kill -> re-route -> answer
        assert s0.stats["transport_failovers"] == 1 and s0.stats["transport_suspects"] == 0
    finally:
        open(stop_path, "w").close()
        s0.close()
        eng.close()
        for p in procs.values():
            p.join(5)
            if p.is_alive():
                p.kill()

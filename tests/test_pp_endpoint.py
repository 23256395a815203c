"""Pipeline endpoint over real sockets on CPU: 2- and 3-stage chains with
the inline, native-engine and gloo-link data planes, K steps in flight,
duplicate answers from the reply cache, failover to another stage-1 replica
(membership event and refused-connect probe), and the ZeroMQ-only path."""
import threading
import time

import pytest
import torch
import torch.distributed as dist

from connex.front_router import EventType
from connex.pp.endpoint import PipelineEndpoint, probe_tcp
from connex.pp.link import Stage0Link, StageWorker
from connex.pp.routing import StaticMembership
from connex.pp.transports import backend_from_env, engine_port
from connex.pp.zmq_base import ZmqStageBase, decode_frames, encode_frames


class Hooks:
    def __init__(self):
        self.held = {}

    def kv_held(self, rid):
        return self.held.get(rid, 0)

    def release(self, rids):
        for r in rids:
            self.held.pop(r, None)

    def reprefill(self, rids):
        pass

    def abort(self, rids):
        pass


def _serve(ep, fn, stop):
    w = StageWorker(ep, Hooks(), lambda td, missing: fn(td))

    def loop():
        while not stop.is_set():
            w.serve_one()
    t = threading.Thread(target=loop, daemon=True)
    t.start()
    return w, t


def _chain(n_stages, data="inline", k=1, replicas=1, **kw):
    mem = StaticMembership(0, 0)
    eps = []
    for s in range(n_stages):
        for r in range(replicas if s > 0 else 1):
            ep = PipelineEndpoint("m", s, n_stages, r, membership=mem, data=data, k=k, recv_timeout_s=1.0, **kw)
            mem.add(s, r, ep.address)
            eps.append(ep)
    return mem, eps


def _add_stage(td, s):
    return {"x": td["x"] + s, "step": td["step"]}


@pytest.mark.parametrize("k", [1, 3])
def test_three_stage_chain_inline(k):
    mem, eps = _chain(3, k=k)
    stop = threading.Event()
    for ep in eps[1:]:
        _serve(ep, lambda td, s=ep.stage_idx: _add_stage(td, s), stop)
    link = Stage0Link(eps[0], Hooks(), recv_timeout_s=2.0)
    try:
        corrs = [link.submit({"x": torch.full((4, 8), float(i)), "step": i}) for i in range(k)]
        for i, c in enumerate(corrs):
            out = link.wait(c)
            assert out["step"] == i and torch.equal(out["x"], torch.full((4, 8), float(i) + 3))
        for i in range(10):
            assert torch.equal(link.step({"x": torch.ones(2, 2), "step": i})["x"], torch.full((2, 2), 4.0))
    finally:
        stop.set()
        for ep in eps:
            ep.close()


def test_duplicate_step_answered_from_cache():
    mem, eps = _chain(2)
    stop = threading.Event()
    w, _ = _serve(eps[1], lambda td: _add_stage(td, 1), stop)
    try:
        c = eps[0].new_step_id()
        eps[0].send_step({"x": torch.zeros(2), "step": 0}, c)
        assert eps[0].recv_step(c, 2.0) is not None
        eps[0]._outstanding.add(c)
        eps[0].send_step({"x": torch.zeros(2), "step": 0}, c)       # a retry under the same corr
        assert eps[0].recv_step(c, 2.0)["x"].tolist() == [1.0, 1.0]
        time.sleep(0.1)
        assert w.stats["steps"] == 1 and eps[1].stats["dedup_replies"] == 1
    finally:
        stop.set()
        for ep in eps:
            ep.close()


def test_failover_to_other_replica_on_event_and_probe():
    mem, eps = _chain(2, replicas=2)
    s0, a, b = eps
    stop_a, stop_b = threading.Event(), threading.Event()
    _serve(a, lambda td: _add_stage(td, 10), stop_a)
    _serve(b, lambda td: _add_stage(td, 20), stop_b)
    link = Stage0Link(s0, Hooks(), recv_timeout_s=1.0)
    try:
        first = link.step({"x": torch.zeros(1), "step": 0})["x"].item()
        victim, other = (a, b) if first == 10 else (b, a)
        # the chosen replica dies; the directory says so -> next step goes to the other one
        (stop_a if victim is a else stop_b).set()
        victim.close()
        mem.emit(EventType.ENDPOINT_DEREGISTERED, 1, victim.replica_idx, reason="killed")
        t0 = time.monotonic()
        out = link.step({"x": torch.zeros(1), "step": 1})["x"].item()
        assert out == (20 if victim is a else 10) and time.monotonic() - t0 < 1.0
        assert s0.stats["failovers"] == 1
        # a dead endpoint refuses TCP connects: the probe confirms it
        assert probe_tcp(victim.address) is False and probe_tcp(other.address) is True
    finally:
        stop_a.set()
        stop_b.set()
        for ep in (s0, other):
            ep.close()


def test_failover_confirmed_by_probe_after_timeout():
    mem, eps = _chain(2, replicas=2)
    s0, a, b = eps
    stops = {a: threading.Event(), b: threading.Event()}
    _serve(a, lambda td: _add_stage(td, 1), stops[a])
    _serve(b, lambda td: _add_stage(td, 1), stops[b])
    link = Stage0Link(s0, Hooks(), recv_timeout_s=0.3)
    try:
        link.step({"x": torch.zeros(1), "step": 0})
        victim = a if s0.current == a.replica_idx else b
        stops[victim].set()
        victim.close()              # no event: only the timeout + refused probe reveal it
        out = link.step({"x": torch.zeros(1), "step": 1})
        assert out["x"].item() == 1.0 and s0.current != victim.replica_idx
    finally:
        for e in stops.values():
            e.set()
        for ep in (s0, a, b):
            if ep is not victim:
                ep.close()


def test_engine_data_plane_one_sided_read():
    from connex_b200.engine import Engine
    e0, e1 = Engine("m", 0, 0, 0, listen_ip="127.0.0.1"), Engine("m", 1, 0, 0, listen_ip="127.0.0.1")
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, membership=mem, data="engine", engine=e0, ring_bytes=1 << 20,
                          recv_timeout_s=2.0)
    s1 = PipelineEndpoint("m", 1, 2, membership=mem, data="engine", engine=e1, ring_bytes=1 << 20,
                          recv_timeout_s=2.0)
    mem.add(0, 0, s0.address)
    mem.add(1, 0, s1.address)
    stop = threading.Event()
    _serve(s1, lambda td: {"h": td["h"] * 2}, stop)
    try:
        link = Stage0Link(s0, Hooks(), recv_timeout_s=2.0)
        for i in range(20):       # 20 x 128 KB through a 1 MB ring: regions come back by CXACK
            h = torch.randn(64, 512)
            assert torch.equal(link.step({"h": h})["h"], h * 2)
        assert s0._ring.awaiting_ack() in (True, False)
    finally:
        stop.set()
        s0.close()
        s1.close()
        e0.close()
        e1.close()


def test_gloo_link_data_plane():
    from connex_b200.parallel.pplink import PairLinks
    store = dist.HashStore()
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, membership=mem, data="link", links=None, recv_timeout_s=5.0)
    s1 = PipelineEndpoint("m", 1, 2, membership=mem, data="link", links=None, recv_timeout_s=5.0)
    s0.links = PairLinks(store, s0.link_id, "cpu", timeout_s=10)
    s1.links = PairLinks(store, s1.link_id, "cpu", timeout_s=10)
    mem.add(0, 0, s0.address)
    mem.add(1, 0, s1.address)
    stop = threading.Event()
    _serve(s1, lambda td: {"h": td["h"] + 1, "tag": td["tag"]}, stop)
    try:
        link = Stage0Link(s0, Hooks(), recv_timeout_s=5.0)
        for i in range(5):
            h = torch.randn(8, 16)
            out = link.step({"h": h, "tag": i})
            assert out["tag"] == i and torch.equal(out["h"], h + 1)
        assert s0.links.get(s1.link_id, tx=True).sent == 5 and s0.links.get(s1.link_id, tx=False).received == 5
    finally:
        stop.set()
        for ep in (s0, s1):
            ep.links.close()
            ep.close()


def test_zmq_only_stage_base_and_frames():
    td = {"a": torch.arange(6.0).view(2, 3), "b": 7, "c": torch.ones(2, dtype=torch.bfloat16)}
    out, ts = decode_frames(encode_frames(td, send_ts=1.5))
    assert ts == 1.5 and out["b"] == 7 and torch.equal(out["a"], td["a"]) and out["c"].dtype == torch.bfloat16
    s0, s1 = ZmqStageBase(0, 2, host="127.0.0.1"), ZmqStageBase(1, 2, host="127.0.0.1")
    try:
        s0.set_peers(forward=s1.router_endpoint)
        s1.set_peers(head=s0.router_endpoint)
        s0.send_tensor_dict(td)
        got = s1.recv_tensor_dict(2000)
        s1.send_tensor_dict({"a": got["a"] * 2})
        assert torch.equal(s0.recv_tensor_dict(2000)["a"], td["a"] * 2)
    finally:
        s0.close()
        s1.close()


def test_backend_selection(monkeypatch):
    monkeypatch.setenv("CONNEX_PP_BACKEND", "connex-rs")
    assert backend_from_env() == "cxengine"
    monkeypatch.setenv("CONNEX_PP_BACKEND", "mooncake")
    with pytest.raises(ValueError, match="cxengine"):
        backend_from_env()
    monkeypatch.setenv("CONNEX_PP_BACKEND", "auto")
    assert backend_from_env(has_cuda=True) == "nccl"
    monkeypatch.delenv("CONNEX_PP_BACKEND")
    assert engine_port(1, 2) == 51201


def test_trace_and_profile_hooks(tmp_path, monkeypatch, caplog):
    import logging
    import connex.pp.endpoint as E
    monkeypatch.setattr(E, "TRACE_PREFIX", str(tmp_path / "tr"))
    monkeypatch.setattr(E, "PROFILE", True)
    monkeypatch.setattr(E, "PROFILE_EVERY", 2)
    mem, eps = _chain(2)
    stop = threading.Event()
    _serve(eps[1], lambda td: _add_stage(td, 1), stop)
    try:
        link = Stage0Link(eps[0], Hooks(), recv_timeout_s=2.0)
        with caplog.at_level(logging.INFO, logger="connex.pp.endpoint"):
            for i in range(4):
                link.step({"x": torch.zeros(2), "step": i})
    finally:
        stop.set()
        for ep in eps:
            ep.close()
    lines = (tmp_path / "tr.stage0.txt").read_text().split("\n")
    events = [ln.split()[2] for ln in lines if ln]
    assert events.count("send_called") == 4 and events.count("recv_done") == 4
    assert (tmp_path / "tr.stage1.txt").read_text().count("arrived") == 4
    assert any("phases" in r.getMessage() for r in caplog.records)


def test_engine_and_process_stats_are_logged(monkeypatch, caplog):
    import logging
    import connex.pp.endpoint as E

    class Eng:
        def stats(self):
            return {"live_peers": 1}
    monkeypatch.setattr(E, "RS_STATS_S", 0.05)
    st = E.process_stats()
    assert st["fds"] > 0 and st["rss_mb"] > 0
    with caplog.at_level(logging.INFO, logger="connex.pp.endpoint"):
        ep = PipelineEndpoint("m", 1, 2, membership=StaticMembership(0, 0), data="inline", engine=Eng())
        time.sleep(0.4)
        ep.close()
    assert any("live_peers" in r.getMessage() and "rss_mb" in r.getMessage() for r in caplog.records)

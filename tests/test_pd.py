"""PD scenario library: KV layouts, heterogeneous-TP plans, producer/consumer
leases over real ZeroMQ with loopback and native-engine planes, group failure."""
import ctypes
import time

import pytest
import torch

from connex.pd.dataplane import CxEnginePlane, LoopbackPlane, resolve_backend
from connex.pd.group import GroupFailureTracker, PeerDeathReporter
from connex.pd.kv_layout import (TensorLayout, block_runs, cx_cache_layouts, find_heads_dims, head_read_ops,
                                 read_ops, register_spans, tensor_layout, tp_plan)
from connex.pd.membership import PD_STAGE, complete_groups, parse_member
from connex.pd.transfer import KVConsumer, KVProducer
from connex.protocol import LogicalEndpointID, PDRole
from tests.helpers import wait_until


# ---- layouts -----------------------------------------------------------------
def test_tensor_layout_kv_first_and_heads():
    t = torch.zeros(2, 10, 16, 8, 128, dtype=torch.bfloat16)  # [2, nb, BS, H, D]
    lo = tensor_layout(t, 10, heads_dims=find_heads_dims(tuple(t.shape), 10, 8, 16))
    assert lo.outer == 2 and lo.seg_bytes == 16 * 8 * 128 * 2 and lo.block_stride == lo.seg_bytes
    assert lo.heads == 8 and lo.tokens == 16 and lo.head_bytes == 256 and not lo.head_major
    hnd = torch.zeros(10, 8, 16, 256, dtype=torch.bfloat16)  # LBHNC
    lo2 = tensor_layout(hnd, 10, heads_dims=find_heads_dims(tuple(hnd.shape), 10, 8, 16, "LBHNC"))
    assert lo2.head_major and lo2.outer == 1
    assert TensorLayout.from_dict(lo2.to_dict()) == lo2
    with pytest.raises(ValueError):
        tensor_layout(torch.zeros(3, 3), 10)


def test_block_runs_and_read_ops():
    assert block_runs([1, 2, 3, 7], [4, 5, 6, 9]) == [(1, 4, 3), (7, 9, 1)]
    lo = TensorLayout(base=1000, outer=2, outer_stride=100000, block_stride=64, seg_bytes=64, num_blocks=100)
    ro = TensorLayout(base=5000, outer=2, outer_stride=200000, block_stride=64, seg_bytes=64, num_blocks=100)
    ops = read_ops([lo], [ro], [1, 2, 3], [10, 11, 12])
    assert ops == [(1000 + 64, 5000 + 640, 192), (101000 + 64, 205000 + 640, 192)]
    bad = TensorLayout(base=0, outer=2, outer_stride=1, block_stride=32, seg_bytes=32, num_blocks=1)
    with pytest.raises(ValueError):
        read_ops([lo], [bad], [1], [1])
    assert register_spans([lo, lo]) == [lo.span]


def test_tp_plan_and_head_reads():
    # prefill TP1 (8 heads) -> decode TP2: each decode rank reads 4 heads from rank 0
    p0, p1 = tp_plan(0, 2, 1, 8), tp_plan(1, 2, 1, 8)
    assert [(s.remote_rank, s.nheads, s.local_head0, s.remote_head0, s.releaser, s.readers) for s in p0] == \
        [(0, 4, 0, 0, True, 2)]
    assert p1[0].remote_head0 == 4 and not p1[0].releaser
    # prefill TP4 -> decode TP1: four sources
    assert [s.remote_rank for s in tp_plan(0, 1, 4, 8)] == [0, 1, 2, 3]
    with pytest.raises(ValueError):
        tp_plan(0, 3, 1, 8)
    # head re-layout between HND caches
    lo = TensorLayout(0, 1, 0, 4 * 16 * 256, 4 * 16 * 256, 4).with_heads(4, 16 * 256, 16, 256, 256)
    ro = TensorLayout(10 ** 6, 1, 0, 8 * 16 * 256, 8 * 16 * 256, 4).with_heads(8, 16 * 256, 16, 256, 256)
    ops = head_read_ops([lo], [ro], [0], [1], 0, 4, 4)
    assert ops == [(0, 10 ** 6 + 8 * 16 * 256 + 4 * 16 * 256, 4 * 16 * 256)]


def test_cx_cache_layouts_match_kernel_layout():
    kv = torch.zeros(3, 2, 5, 8, 16, 128, dtype=torch.bfloat16)
    los = cx_cache_layouts(kv)
    assert len(los) == 3 and los[0].outer == 2 and los[0].head_major
    assert los[1].base - los[0].base == kv.stride(0) * 2


# ---- producer / consumer -------------------------------------------------------
def _host_cache(nb=32, seg=4096, fill=0):
    buf = (ctypes.c_char * (2 * nb * seg))()
    if fill:
        ctypes.memset(buf, fill, len(buf))
    lo = TensorLayout(base=ctypes.addressof(buf), outer=2, outer_stride=nb * seg, block_stride=seg, seg_bytes=seg,
                      num_blocks=nb)
    return buf, lo


def _fill_blocks(buf, lo, blocks, tag):
    for b in blocks:
        for o in range(2):
            off = o * lo.outer_stride + b * lo.block_stride
            ctypes.memset(ctypes.addressof(buf) + off, (tag + b + o) % 250 + 1, lo.seg_bytes)


def _block(buf, lo, b, o=0):
    off = o * lo.outer_stride + b * lo.block_stride
    return bytes(buf)[off:off + lo.seg_bytes]


def _wait_done(cons, n=1, timeout=5.0):
    out = []
    deadline = time.time() + timeout
    while len(out) < n and time.time() < deadline:
        out += cons.take_done()
        time.sleep(0.005)
    return out


def test_hold_acquire_pull_release_loopback():
    pbuf, plo = _host_cache()
    dbuf, dlo = _host_cache()
    prod = KVProducer(LoopbackPlane(), [plo], bind_ip="127.0.0.1", retain_s=30, block_size=16)
    cons = KVConsumer(LoopbackPlane(), [dlo], block_size=16)
    try:
        _fill_blocks(pbuf, plo, [3, 4, 5], 7)
        prod.hold("req1", "tid1", [3, 4, 5])
        cons.pull("req1", f"127.0.0.1:{prod.port}", "tid1", [10, 11, 20])
        res = _wait_done(cons)
        assert res and res[0].ok and res[0].nbytes == 3 * 2 * 4096
        for lb, rb in ((10, 3), (11, 4), (20, 5)):
            assert _block(dbuf, dlo, lb, 1) == _block(pbuf, plo, rb, 1)
        # a second decode instance can re-pull while the hold lives (decode death)
        cons.pull("req1", f"127.0.0.1:{prod.port}", "tid1", [1, 2], first_block=1)
        assert _wait_done(cons)[0].ok
        cons.release(f"127.0.0.1:{prod.port}", "tid1")
        assert wait_until(lambda: "req1" in prod.take_finished() or prod.held() == 0, 3)
        # released: acquire now fails (reported, not raised)
        cons.pull("req1", f"127.0.0.1:{prod.port}", "tid1", [1])
        r = _wait_done(cons)[0]
        assert not r.ok and "unknown" in r.why
    finally:
        cons.close()
        prod.close()


def test_lease_expiry_unknown_retry_and_stale_release():
    pbuf, plo = _host_cache()
    dbuf, dlo = _host_cache()
    prod = KVProducer(LoopbackPlane(), [plo], bind_ip="127.0.0.1", retain_s=0.2)
    cons = KVConsumer(LoopbackPlane(), [dlo], acquire_wait_s=1.0, who="decodeA")
    addr = f"127.0.0.1:{prod.port}"
    try:
        # acquire arrives before the hold: retried until the hold shows up
        cons.pull("r", addr, "t", [0])
        time.sleep(0.05)
        prod.hold("r", "t", [1])
        assert _wait_done(cons)[0].ok
        # stale release from another owner is ignored (single reader)
        assert cons.control(addr, {"op": "release", "tid": "t", "who": "someone-else"})["stale"]
        assert prod.held() == 1
        time.sleep(0.3)
        assert "r" in prod.take_finished() and prod.stats["expired"] == 1
        # release before hold: the hold is dropped on arrival
        cons.control(addr, {"op": "release", "tid": "t2", "who": "x"})
        prod.hold("r2", "t2", [2])
        assert prod.held() == 0 and "r2" in prod.take_finished()
        # multi-reader release (heterogeneous TP): freed after all readers
        prod.hold("r3", "t3", [3])
        assert cons.control(addr, {"op": "release", "tid": "t3", "who": "a", "of": 2})["pending"] == 1
        assert cons.control(addr, {"op": "release", "tid": "t3", "who": "b", "of": 2}) == {"ok": True}
        assert prod.held() == 0
        assert cons.control(addr, {"op": "ping"})["ok"]
    finally:
        cons.close()
        prod.close()


def test_producer_unreachable_and_outside_registered_memory():
    dbuf, dlo = _host_cache()
    cons = KVConsumer(LoopbackPlane(), [dlo], ctrl_timeout_ms=200)
    cons.pull("r", "127.0.0.1:1", "t", [0])
    r = _wait_done(cons)[0]
    assert not r.ok and r.why == "producer unreachable"
    pbuf, plo = _host_cache(nb=64)
    prod = KVProducer(LoopbackPlane(), [plo], bind_ip="127.0.0.1")
    prod.hold("r", "t", [1])
    cons.pull("r", f"127.0.0.1:{prod.port}", "t", [40])  # block 40 is outside our 32-block cache
    r = _wait_done(cons)[0]
    assert not r.ok and "outside" in r.why
    cons.close()
    prod.close()


def test_cxengine_plane_pull_between_two_engines():
    pbuf, plo = _host_cache()
    dbuf, dlo = _host_cache()
    pp = CxEnginePlane("m", PD_STAGE[PDRole.PREFILL], 0, 0)
    dp = CxEnginePlane("m", PD_STAGE[PDRole.DECODE], 0, 0)
    prod = KVProducer(pp, [plo], bind_ip="127.0.0.1")
    cons = KVConsumer(dp, [dlo])
    try:
        _fill_blocks(pbuf, plo, [0, 1, 2, 9], 3)
        prod.hold("q", "tq", [0, 1, 2, 9])
        cons.pull("q", f"127.0.0.1:{prod.port}", "tq", [5, 6, 7, 8])
        assert _wait_done(cons)[0].ok
        assert _block(dbuf, dlo, 8, 1) == _block(pbuf, plo, 9, 1)
    finally:
        cons.close()
        prod.close()
        pp.close()
        dp.close()


def test_backend_resolution():
    assert resolve_backend("connex-rs") == "cxengine" and resolve_backend("mooncake") == "cxengine"
    assert resolve_backend("loopback") == "loopback" and resolve_backend("nvlink") == "nvlink"
    with pytest.raises(ValueError):
        resolve_backend("bogus")


# ---- group failure / membership ---------------------------------------------------
def test_group_failure_tracker_rules():
    t = GroupFailureTracker("m", [1000])
    assert t.on_event({"type": "failed", "peer": ("m", 1000, 0, 1)}) is None  # never up
    t.on_event({"type": "up", "peer": ("m", 1000, 0, 1)})
    assert t.on_event({"type": "failed", "peer": ("m", 1000, 0, 1), "reason": "heartbeat timeout"}) is None
    lid = t.on_event({"type": "failed", "peer": ("m", 1000, 0, 1), "reason": "connection lost"})
    assert lid == LogicalEndpointID("m", 1000, 0, 1)
    assert t.on_event({"type": "failed", "peer": ("m", 1000, 0, 1)}) is None  # reported once
    assert t.on_event({"type": "up", "peer": ("x", 1000, 0, 1)}) is None      # other model


def test_peer_death_reporter_with_engine_events():
    from connex_b200.engine import Engine
    got = []
    b = Engine("m", 1001, 0, 0, listen_ip="127.0.0.1")
    a = Engine("m", 1000, 1, 2, listen_ip="127.0.0.1")
    rep = PeerDeathReporter(b, "tcp://unused:1", "m", report=lambda lid, why: got.append((lid, why)))
    rep.start()
    assert b.connect(a.local_url)
    time.sleep(0.2)
    a.close()
    assert wait_until(lambda: got, 3)
    assert got[0][0] == LogicalEndpointID("m", 1000, 1, 2) and "peer died" in got[0][1]
    rep.stop()
    b.close()


def test_complete_groups_and_parse():
    r = lambda shard, rep, g, addrs: {"lid": {"model_name": "m", "stage_idx": 1000, "shard_idx": shard,
                                              "replica_idx": rep}, "addresses": addrs, "state": 1,
                                      "group_size": g}
    routes = [r(0, 0, 2, ["http://a:1", "kv=a:2"]), r(1, 0, 2, ["tp"]), r(0, 1, 2, ["http://b:1"]),
              r(0, 2, 1, ["http://c:1", "rs=c:3"])]
    groups = complete_groups(routes)
    assert [g["lid"]["replica_idx"] for g in groups] == [2, 0]
    m = parse_member(groups[1])
    assert m.url == "http://a:1" and m.kv_addr == "a:2" and m.group_size == 2 and m.role == PDRole.PREFILL
    assert parse_member(groups[0]).extra == ["rs=c:3"]


def test_pd_member_pools_through_front_router():
    from connex.front_router import FrontRouter, FrontRouterConfig
    from connex.pd.membership import PDMember, fetch_pools, report_failure
    from tests.helpers import free_ports
    p1, p2 = free_ports(2)
    fr = FrontRouter(FrontRouterConfig(f"tcp://127.0.0.1:{p1}", f"tcp://127.0.0.1:{p2}"))
    fr.start()
    api, ev = f"tcp://127.0.0.1:{p1}", f"tcp://127.0.0.1:{p2}"
    members = [PDMember(api, "m", PDRole.PREFILL, 0, "http://p0:1", kv_addr="p0:9", events=ev),
               PDMember(api, "m", PDRole.DECODE, 0, "http://d0:1", events=ev, shard=0, group_size=2),
               PDMember(api, "m", PDRole.DECODE, 0, "http://d0:1", events=ev, shard=1, group_size=2)]
    try:
        for m in members:
            assert m.start()
        pools = fetch_pools(api, "m")
        assert [x.url for x in pools[PDRole.PREFILL]] == ["http://p0:1"]
        assert [x.url for x in pools[PDRole.DECODE]] == ["http://d0:1"]
        # one TP rank of the decode group dies -> the whole group leaves the pool
        failed = report_failure(api, LogicalEndpointID("m", PD_STAGE[PDRole.DECODE], 1, 0), "test")
        assert len(failed) == 2
        assert fetch_pools(api, "m")[PDRole.DECODE] == []
    finally:
        for m in members:
            m.client.kill()
        fr.stop()

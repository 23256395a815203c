"""Pipeline step protocol: wire format, dedupe/stale rules, handover, ring, routing, drivers."""
import struct
import threading
import time

import pytest

from connex.pp import wire
from connex.pp.handover import (CX_CTX, CX_MISSING, FINISHED, REQUEST_IDS, FinishedOutbox, KVLedger,
                                RewindBudget, blank_rows, find_missing, merge_missing)
from connex.pp.link import Stage0Link, StageWorker, StepFailed
from connex.pp.ring import RegionTable
from connex.pp.routing import Lid, Route, StaticMembership, select_peer
from connex.pp.steps import CorrFilter, ReplyCache, StepIds
from connex.pp.testing import LoopbackTransferEngine, fake_chain


# ---- wire ------------------------------------------------------------------------
def test_signal_golden_bytes():
    sig = wire.encode_signal(0x1122334455667788, 4096, b"10.0.0.1:5000", 0xAABBCCDD00000007, b"")
    assert sig[:8] == b"CONNEXTE"
    assert sig[8:28] == struct.pack("!QQI", 0x1122334455667788, 4096, 13)
    assert sig[28:41] == b"10.0.0.1:5000"
    assert sig[41:49] == struct.pack("!Q", 0xAABBCCDD00000007)
    s = wire.decode_signal(sig)
    assert (s.src_ptr, s.total, s.url, s.corr, s.tail) == (0x1122334455667788, 4096, "10.0.0.1:5000",
                                                          0xAABBCCDD00000007, b"")
    assert wire.signal_corr(sig) == 0xAABBCCDD00000007
    # legacy sender without a correlation id
    old = wire.WIRE_MAGIC + struct.pack("!QQI", 1, 2, 3) + b"abc"
    assert wire.decode_signal(old).corr is None
    with pytest.raises(ValueError):
        wire.decode_signal(b"NOTMAGIC" + b"\0" * 20)


def test_g2_layout_roundtrip_and_bytes():
    layout = [("hidden_states", "bfloat16", (64, 4096), 0, 64 * 4096 * 2),
              ("residual", "bfloat16", (64, 4096), wire.align(64 * 4096 * 2), 64 * 4096 * 2)]
    lb = wire.encode_layout(layout)
    assert lb[:2] == struct.pack("!H", 2)
    assert lb[2:6] == struct.pack("!HBB", len("hidden_states"), wire.DT_CODE["bfloat16"], 2)
    assert wire.decode_layout(lb) == layout
    g2 = wire.encode_g2(7, lb, b"tcp://a:1", b"tcp://o:2", b"NT")
    assert g2[:2] == b"G2"
    tok, lb2, ack, origin, nt = wire.decode_g2(g2[2:])
    assert (tok, lb2, ack, origin, nt) == (7, lb, "tcp://a:1", "tcp://o:2", b"NT")
    assert wire.encode_layout([("x", "complex64", (1,), 0, 8)]) is None
    assert wire.DT_NAMES[:3] == ("float32", "float16", "bfloat16")  # append-only codes


def test_layout_codec_cache_and_alignment():
    c = wire.LayoutCodec(cap=2)
    key = (("a", "float32", (3,)), ("b", "int64", (5,)))
    layout, total, lb = c.layout_for(key, [12, 40])
    assert layout[1][3] == 256 and total == 512
    assert c.layout_for(key, [12, 40])[2] is lb
    assert c.parse(lb) == layout


def test_ack_and_corr():
    a = wire.encode_ack(0xDEAD)
    assert a == b"CXACK" + struct.pack("!Q", 0xDEAD)
    assert wire.decode_ack(a) == 0xDEAD and wire.decode_ack(b"junk") is None
    c = wire.make_corr(0x1234, 99)
    assert wire.corr_incarnation(c) == 0x1234 and wire.corr_seq(c) == 99


# ---- steps -----------------------------------------------------------------------
def test_corr_filter_window():
    f = CorrFilter(window=1)
    assert f.accept(wire.make_corr(1, 5)) and not f.accept(wire.make_corr(1, 4))
    assert f.accept(wire.make_corr(2, 1))  # another incarnation
    assert f.accept(None) and f.accept(0)
    f4 = CorrFilter(window=4)
    assert f4.accept(wire.make_corr(1, 10))
    assert f4.accept(wire.make_corr(1, 7))      # inside the window (out-of-order retry)
    assert not f4.accept(wire.make_corr(1, 6))  # 4 behind -> stale


def test_step_ids_and_reply_cache():
    ids = StepIds(base=5 << 32)
    assert [ids.next(), ids.next()] == [(5 << 32) + 1, (5 << 32) + 2]
    evicted = []
    rc = ReplyCache(k=2, on_evict=evicted.append)
    rc.put(1, "a")
    rc.put(2, "b")
    rc.put(3, "c")
    assert evicted == ["a"] and 2 in rc and len(rc) == 2
    rc.put(3, "c2")
    assert evicted == ["a", "c"] and rc.get(3) == "c2"


# ---- handover --------------------------------------------------------------------
def test_handover_rules():
    held = {"r1": 10, "r2": 0}.get
    assert find_missing(["r1", "r2", "r3"], [10, 5, 0], lambda r: held(r, 0)) == ["r2"]
    assert find_missing(["r1"], None, lambda r: 0) == []
    assert merge_missing(["a"], ["b", "a"]) == ["a", "b"] and merge_missing(None, None) is None
    assert blank_rows([[1], [2]], ["a", "b"], ["b"]) == [[1], []]
    led = KVLedger()
    led.commit(["a", "b"], [0, 4], [5, 1], missing=["b"])
    assert led.kv_held("a") == 5 and led.kv_held("b") == 0
    led.commit(["a"], [2], [1])  # re-executed older step never shrinks
    assert led.kv_held("a") == 5
    ob = FinishedOutbox(repeat=2)
    ob.add(["x"])
    assert ob.take() == ["x"] and ob.take() == ["x"] and ob.take() is None
    rb = RewindBudget(max_rewinds=1)
    assert rb.split(["q"]) == (["q"], []) and rb.split(["q"]) == ([], ["q"])


# ---- ring ------------------------------------------------------------------------
def test_region_table_ack_pin_and_deadline():
    rt = RegionTable(1000, token_base=1 << 32)
    a = rt.alloc(400, now=0, hold_s=5, want_ack=True)
    b = rt.alloc(400, now=0, hold_s=5, want_ack=True)
    assert a[0] == 0 and b[0] == 400
    assert rt.alloc(400, now=0, hold_s=5, want_ack=True) is None  # wraps onto busy region a
    rt.ack(a[1])
    c = rt.alloc(400, now=0, hold_s=5, want_ack=True)
    assert c is not None and c[0] == 0
    rt.pin(c[1])
    rt.ack(c[1])
    assert rt.alloc(400, now=10, hold_s=5, want_ack=True) is not None  # b expired
    assert rt.alloc(400, now=10, hold_s=5, want_ack=True) is None or True
    tok = rt.add_temp("tmpbuf", now=0, hold_s=1, want_ack=True)
    assert "tmpbuf" in rt.collect(now=2) and rt.expired_unacked >= 1
    assert rt.alloc(5000, now=0, hold_s=1, want_ack=False) is None


# ---- routing ---------------------------------------------------------------------
def _routes(*specs):
    return [Route(Lid(s, r), [a]) for s, r, a in specs]


def test_select_peer_rules():
    peers = _routes((1, 0, "h:1"), (1, 1, "h:2"), (0, 0, "h:0"), (0, 1, "h:9"))
    assert select_peer(peers, 1, 0, 1, None, set()) == ("h:2", 1, True)  # rank based
    assert select_peer(peers, 1, 0, 0, 1, set()) == ("h:2", 1, False)    # sticky current
    assert select_peer(peers, 1, 0, 0, None, {(1, 0)}) == ("h:2", 1, True)  # departed skipped
    assert select_peer(peers, 1, 0, 0, None, set(), exclude_replica=0) == ("h:2", 1, True)
    amb = _routes((1, 0, "x:1"), (2, 0, "x:1"), (1, 1, "h:2"))
    assert select_peer(amb, 1, 0, 0, None, set())[0] == "h:2"  # ambiguous address dropped
    assert select_peer(_routes((2, 0, "a:1")), 1, 0, 0, None, set()) == (None, None, False)


def test_static_membership_events():
    m = StaticMembership(0)
    got = []
    m.on_event("dereg", lambda e: got.append(e.payload["lid"]))
    m.add(1, 0, "h:1")
    assert len(m.get_stage_peers(1)) == 1
    m.remove(1, 0)
    m.emit("dereg", 1, 0, reason="x")
    assert got == [{"stage_idx": 1, "replica_idx": 0}] and m.get_stage_peers(1) == []


# ---- drivers over the in-process chain -------------------------------------------
class Hooks:
    def __init__(self):
        self.ledger = KVLedger()
        self.released, self.reprefilled, self.aborted = [], [], []

    def kv_held(self, rid):
        return self.ledger.kv_held(rid)

    def release(self, rids):
        self.released += list(rids)
        self.ledger.forget(rids)

    def reprefill(self, rids):
        self.reprefilled += list(rids)

    def abort(self, rids):
        self.aborted += list(rids)


def _serve(worker, stop):
    while not stop.is_set():
        worker.serve_one()


def _chain_with_workers(n, k=1):
    links = fake_chain(n, k)
    hooks = [Hooks() for _ in links]
    stop = threading.Event()
    workers = []
    for i in range(1, n):
        h = hooks[i]
        w = StageWorker(links[i], h, lambda td, miss, i=i: {"x": td.get("x", 0) + 1},
                        commit=lambda td, miss, h=h: h.ledger.commit(td.get(REQUEST_IDS), td.get(CX_CTX),
                                                                     missing=miss))
        th = threading.Thread(target=_serve, args=(w, stop), daemon=True)
        th.start()
        workers.append((w, th))
    return links, hooks, stop, workers


def test_stage0_link_steps_and_duplicate_dedupe():
    links, hooks, stop, workers = _chain_with_workers(3, k=2)
    s0 = Stage0Link(links[0], hooks[0], recv_timeout_s=0.5)
    r = s0.step({"x": 1}, ["a"], [0])
    assert r["x"] == 3
    links[1].inbox.dup_next = 1  # duplicated forward message: answered from cache
    r = s0.step({"x": 10}, ["a"], [1])
    assert r["x"] == 12
    assert links[1].computed == 2
    stop.set()


def test_stage0_retry_after_drop_and_k_in_flight():
    links, hooks, stop, workers = _chain_with_workers(2, k=4)
    s0 = Stage0Link(links[0], hooks[0], recv_timeout_s=0.1)
    links[1].inbox.drop_next = 1
    corrs = [s0.submit({"x": i}, ["a"], [i]) for i in range(4)]
    outs = [s0.wait(c)["x"] for c in corrs]
    assert outs == [1, 2, 3, 4] and s0.stats["retries"] >= 1
    stop.set()


def test_failover_missing_kv_reprefill():
    """Replica dies: stage 0 fails over to a fresh replica that holds no KV ->
    cx_missing -> re-prefill on stage 0."""
    links, hooks, stop, workers = _chain_with_workers(2, k=1)
    s0 = Stage0Link(links[0], hooks[0], recv_timeout_s=0.1, max_attempts=3)
    s0.step({"x": 0}, ["a"], [0])          # prefill on replica A
    # new replica B
    from connex.pp.testing import FakeLink
    b = FakeLink(1, 2, 1)
    b.head = links[0]
    hb = Hooks()
    wb = StageWorker(b, hb, lambda td, miss: {"x": -1},
                     commit=lambda td, miss: hb.ledger.commit(td.get(REQUEST_IDS), td.get(CX_CTX), missing=miss))
    stop_b = threading.Event()
    threading.Thread(target=_serve, args=(wb, stop_b), daemon=True).start()
    links[1].inbox.dead = True
    links[1].healthy = False
    links[0].fail_over(b)
    r = s0.step({"x": 5}, ["a"], [7])      # a decode step: B lacks the 7 tokens
    assert r["__cx_reprefilled__"] == ["a"] and hooks[0].reprefilled == ["a"] and hb.released == ["a"]
    stop.set()
    stop_b.set()


def test_step_failed_when_downstream_dead():
    links, hooks, stop, workers = _chain_with_workers(2)
    links[1].inbox.dead = True
    links[1].healthy = False
    s0 = Stage0Link(links[0], hooks[0], recv_timeout_s=0.05, max_attempts=2)
    with pytest.raises(StepFailed):
        s0.step({"x": 1})
    stop.set()


def test_finished_ids_piggyback_and_release():
    links, hooks, stop, workers = _chain_with_workers(2)
    s0 = Stage0Link(links[0], hooks[0], recv_timeout_s=0.5)
    s0.step({"x": 1}, ["a", "b"], [0, 0])
    s0.finished(["b"])
    s0.step({"x": 1}, ["a"], [1])
    assert wait_released(hooks[1], "b")
    stop.set()


def wait_released(h, rid, timeout=2.0):
    deadline = time.time() + timeout
    while time.time() < deadline:
        if rid in h.released:
            return True
        time.sleep(0.01)
    return False


def test_loopback_engine_read():
    a, b = LoopbackTransferEngine("a:1"), LoopbackTransferEngine("b:1")
    pa, pb = a.allocate_managed_buffer(64), b.allocate_managed_buffer(64)
    a.write_bytes_to_buffer(pa, b"hello", 5)
    assert b.transfer_sync_read("a:1", pb, pa, 5) == 0
    assert b.read_bytes_from_buffer(pb, 5) == b"hello"
    assert b.transfer_sync_read("nope:1", pb, pa, 5) == -1

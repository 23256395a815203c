"""Edge cases of the control plane and the serving layer on CPU: an aborted
migration cannot be cut over and a completed one is not replayed; pool admin
needs loopback or the admin token; a stream that breaks after its last token
is a success and is not resumed; a lapsed
blacklist re-arms the replica without a prober; a stale release from an
earlier reader does not free a newer reader's KV hold."""
import asyncio
import ctypes
import types

from connex.front_router import EventBus, EpochManager, LogicalEndpointID, MigrationOrchestrator, RouteManager
from connex.pd.dataplane import LoopbackPlane
from connex.pd.kv_layout import TensorLayout
from connex.pd.transfer import KVProducer
from connex.serving.fake_backend import FakeBackend, reference
from connex.serving.pd_router import ElasticPool, PDRouter
from connex.serving.proxy import Pool
from tests.helpers import free_ports
from tests.test_serving import _proxy, _run, _serve, _stream, _text


def _orchestrator():
    rm, em = RouteManager(), EpochManager()
    bus = EventBus(f"tcp://127.0.0.1:{free_ports(1)[0]}")
    bus.start()
    lid = LogicalEndpointID("m", 1, 0, 0)
    rm.add_route(lid, ["tcp://a:1"], [], 0)
    return MigrationOrchestrator(rm, em, bus), rm, bus, lid


def test_aborted_migration_cannot_be_cut_over_and_cutover_is_not_replayed():
    mo, rm, bus, lid = _orchestrator()
    try:
        m = mo.prepare_migration(lid, "tcp://b:2")
        assert mo.abort_migration(m.migration_id, "shadow failed")
        assert mo.execute_cutover(m.migration_id) is False
        assert rm.get_route(lid).addresses == ["tcp://a:1"]
        m2 = mo.prepare_migration(lid, "tcp://c:3")
        assert mo.execute_cutover(m2.migration_id) is True
        assert rm.get_route(lid).addresses == ["tcp://c:3"]
        assert mo.execute_cutover(m2.migration_id) is False           # not replayed
        assert mo.abort_migration(m2.migration_id, "late") is False
    finally:
        bus.stop()


def test_pool_admin_needs_loopback_or_the_token():
    r = PDRouter(ElasticPool([], probe_new=False), ElasticPool([], probe_new=False), probe_interval=0)
    req = lambda remote, auth="": types.SimpleNamespace(remote=remote, headers={"Authorization": auth})
    assert r._admin_allowed(req("127.0.0.1")) and r._admin_allowed(req("::1"))
    assert not r._admin_allowed(req("10.1.2.3"))
    r.admin_token = "s3cret"
    assert r._admin_allowed(req("10.1.2.3", "Bearer s3cret"))
    assert not r._admin_allowed(req("10.1.2.3", "Bearer wrong"))


def test_break_after_the_last_token_is_success():
    async def main():
        a, b = FakeBackend(), FakeBackend()
        ua, ub = await a.start(), await b.start()
        a.fail, a.fail_count = ("reset", 5), 1
        b.fail, b.fail_count = ("reset", 5), 1
        p = _proxy([ua, ub])
        pr, url = await _serve(p.app())
        try:
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t2 t3", "max_tokens": 5})
            assert done and _text(chunks) == reference("t2 t3", 5)[1]
            assert len(a.requests) + len(b.requests) == 1 and p.stats["resumes"] == 0
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_lapsed_blacklist_rearms_the_replica_without_a_prober():
    async def main():
        pool = Pool(["http://x:1", "http://y:2"], blacklist_s=0.05)
        ep = pool.eps["http://x:1"]
        pool.mark_bad(ep, "test")
        assert ep.dead.is_set() and pool.pick(exclude=["http://y:2"]) is ep     # last resort
        await asyncio.sleep(0.08)
        assert pool.pick(exclude=["http://y:2"]) is ep and not ep.dead.is_set() and ep.bad_until == 0
    _run(main())


def test_stale_release_does_not_free_a_newer_readers_hold():
    buf = (ctypes.c_char * (2 * 8 * 256))()
    lo = TensorLayout(base=ctypes.addressof(buf), outer=2, outer_stride=8 * 256, block_stride=256, seg_bytes=256,
                      num_blocks=8)
    prod = KVProducer(LoopbackPlane(), [lo], bind_ip="127.0.0.1", retain_s=30)
    try:
        prod.hold("r", "t", [1, 2])
        assert prod.answer({"op": "acquire", "tid": "t", "who": "old"})["ok"]
        assert prod.answer({"op": "acquire", "tid": "t", "who": "new"})["ok"]    # a re-pull by a new decode
        assert prod.answer({"op": "release", "tid": "t", "who": "old"}).get("stale") is True
        assert prod.held() == 1
        assert prod.answer({"op": "release", "tid": "t", "who": "new"}) == {"ok": True}
        assert prod.held() == 0 and "r" in prod.take_finished()
    finally:
        prod.close()

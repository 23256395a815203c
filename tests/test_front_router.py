"""Front router and EPC client over real ZeroMQ on localhost: route expiry by
lease (pure logic and live), event-synced route caches with sequence gaps,
stage queries, migration (prepare -> shadow ready -> cutover), address
updates, fallback routes, and TP groups failing as one endpoint."""
import time

import pytest

from connex.epc_client import EPCV2Client, EPCV2ClientConfig
from connex.front_router import (EventType, FrontRouter, FrontRouterConfig, LogicalEndpointID, MemberManager,
                                 RouteManager, RouteState)
from tests.helpers import free_ports, wait_until


@pytest.fixture
def fr():
    api, ev = free_ports(2)
    r = FrontRouter(FrontRouterConfig(f"tcp://127.0.0.1:{api}", f"tcp://127.0.0.1:{ev}", heartbeat_timeout_s=0.4,
                                      grace_period_s=0.4, check_interval_s=0.05))
    r.start()
    r.urls = (f"tcp://127.0.0.1:{api}", f"tcp://127.0.0.1:{ev}")
    yield r
    r.stop()


def _client(fr, stage, replica=0, addr=None, shard=0, group=1, hb=0.05):
    c = EPCV2Client(EPCV2ClientConfig(front_router_api=fr.urls[0], front_router_events=fr.urls[1], model_name="m",
                                      stage_idx=stage, shard_idx=shard, replica_idx=replica, group_size=group,
                                      local_addresses=[addr or f"tcp://10.0.0.{stage}:{5000 + replica}"],
                                      heartbeat_interval_s=hb, ucx_enabled=False))
    assert c.start()
    return c


def _lid(stage, replica=0, shard=0):
    return LogicalEndpointID("m", stage, shard, replica)


def test_route_manager_expiry_is_ordered_by_heartbeat():
    rm = RouteManager()
    for rep in range(3):
        rm.add_route(_lid(1, rep), [f"a{rep}"], [], 0)
    now = time.time()
    time.sleep(0.3)
    rm.heartbeat(_lid(1, 2))                             # only replica 2 is fresh
    unhealthy, removed = rm.collect_expired(1.0, 1.0, now=now + 1.1)
    assert sorted(r.lid.replica_idx for r in unhealthy) == [0, 1] and not removed
    assert rm.get_route(_lid(1, 0)).state == RouteState.UNHEALTHY
    known, recovered = rm.heartbeat(_lid(1, 0))           # heartbeats again: back to ACTIVE
    assert known and recovered and rm.get_route(_lid(1, 0)).state == RouteState.ACTIVE
    unhealthy, removed = rm.collect_expired(1.0, 1.0, now=now + 3.0)
    assert [r.lid.replica_idx for r in removed] == [1] and rm.get_route(_lid(1, 1)) is None
    assert rm.heartbeat(_lid(9)) == (False, False)


def test_lease_settings_from_the_environment(monkeypatch):
    monkeypatch.setenv("CONNEX_HEARTBEAT_TIMEOUT_S", "0.8")
    monkeypatch.setenv("CONNEX_UNHEALTHY_GRACE_S", "2")
    mm = MemberManager(RouteManager())
    assert (mm.HEARTBEAT_TIMEOUT_S, mm.GRACE_PERIOD_S) == (0.8, 2.0) and mm.check_interval_s == pytest.approx(0.2)
    monkeypatch.setenv("CONNEX_HEARTBEAT_TIMEOUT_S", "bogus")
    assert MemberManager(RouteManager()).HEARTBEAT_TIMEOUT_S == 3.0


def test_registration_events_keep_caches_in_sync(fr):
    a = _client(fr, 0)
    seen = []
    a.on_event(EventType.ENDPOINT_REGISTERED, lambda e: seen.append(e.payload["lid"]["replica_idx"]))
    try:
        assert wait_until(a.cache_in_sync, 3)
        b1, b2 = _client(fr, 1, 0), _client(fr, 1, 1)
        assert wait_until(lambda: len(a.get_stage_peers(1, refresh="never")) == 2, 3)
        # both registrations arrive as events (under load a snapshot reload may absorb one of them)
        assert wait_until(lambda: seen == [0, 1], 3) and a.stats["incremental_applied"] >= 1
        assert [r.lid.replica_idx for r in a.query_stage_routes(1)] == [0, 1]
        b2.stop()                                          # graceful: deregistered at once
        assert wait_until(lambda: len(a.get_stage_peers(1, refresh="never")) == 1, 3)
        b1.stop()
    finally:
        a.stop()


def test_sequence_gap_forces_a_full_refresh(fr):
    a = _client(fr, 0)
    try:
        assert wait_until(a.cache_in_sync, 3)
        b = _client(fr, 1)
        assert wait_until(lambda: len(a.get_stage_peers(1, refresh="never")) == 1, 3)
        a.route_table.seq -= 5                             # pretend events were lost
        c = _client(fr, 1, 1)
        assert wait_until(lambda: a.stats["seq_gaps"] >= 1 and len(a.get_stage_peers(1, refresh="never")) == 2, 3)
        assert a.stats["full_refreshes"] >= 1 and wait_until(a.cache_in_sync, 3)
        b.stop()
        c.stop()
    finally:
        a.stop()


def test_dead_member_is_unhealthy_then_removed_and_recovery_is_announced(fr):
    a = _client(fr, 0)
    events = []
    for t in (EventType.ENDPOINT_UNHEALTHY, EventType.ENDPOINT_DEREGISTERED, EventType.ENDPOINT_REGISTERED):
        a.on_event(t, lambda e, t=t: events.append((t, e.payload["lid"]["replica_idx"], e.payload.get("reason"))))
    try:
        b = _client(fr, 1, 0)
        c = _client(fr, 1, 1)
        assert wait_until(lambda: len(a.get_stage_peers(1, refresh="never")) == 2, 3)
        t0 = time.monotonic()
        b.kill()                                           # no deregister: only the lease tells
        assert wait_until(lambda: (EventType.ENDPOINT_DEREGISTERED, 0, "expired") in events, 3)
        assert time.monotonic() - t0 < 2.0
        assert (EventType.ENDPOINT_UNHEALTHY, 0, None) in events
        assert [r.lid.replica_idx for r in a.get_stage_peers(1, refresh="always")] == [1]
        # a member that missed its lease briefly and heartbeats again is announced as recovered
        recovered = []
        a.on_event(EventType.ENDPOINT_REGISTERED, lambda e: e.payload.get("recovered") and recovered.append(1))
        fr.route_manager.update_route_state(_lid(1, 1), RouteState.UNHEALTHY)
        assert wait_until(lambda: bool(recovered), 3)
        assert fr.route_manager.get_route(_lid(1, 1)).state == RouteState.ACTIVE
        c.stop()
    finally:
        a.stop()


def test_migration_prepare_shadow_cutover(fr):
    a = _client(fr, 0)
    done = []
    a.on_event(EventType.CUTOVER_COMPLETE, lambda e: done.append(e.payload))
    try:
        b = _client(fr, 1, addr="tcp://10.0.0.1:5000")
        assert wait_until(lambda: len(a.get_stage_peers(1, refresh="never")) == 1, 3)
        e0 = a.call("get_epoch", {})["epoch"]
        r = a.call("prepare_migration", {"lid": _lid(1).to_dict(), "new_address": "tcp://10.0.0.9:6000"})
        assert r["success"] and r["new_epoch"] > e0
        mid = r["migration_id"]
        # clients got PREPARE_MIGRATION and answered shadow_ready on their own
        assert wait_until(lambda: fr.migration_orchestrator.get(mid) is not None and
                          len(fr.migration_orchestrator.get(mid).shadows_ready) >= 1, 3)
        assert a.call("execute_cutover", {"migration_id": mid})["success"]
        assert wait_until(lambda: bool(done), 3)
        assert wait_until(lambda: a.get_peer_address(_lid(1)) == "tcp://10.0.0.9:6000", 3)
        assert a.call("get_epoch", {})["epoch"] >= r["new_epoch"]
        b.stop()
    finally:
        a.stop()


def test_address_update_and_fallback_route(fr):
    a = _client(fr, 0)
    try:
        b0, b1 = _client(fr, 1, 0), _client(fr, 1, 1)
        assert b0.update_my_address(["tcp://10.1.1.1:7000"])
        assert wait_until(lambda: a.get_peer_address(_lid(1, 0)) == "tcp://10.1.1.1:7000", 3)
        fr.route_manager.update_route_state(_lid(1, 0), RouteState.DRAINING)
        got = a.call("get_route", {"lid": _lid(1, 0).to_dict()})
        assert got["is_fallback"] and got["fallback_replica"] == 1
        strict = a.call("get_route", {"lid": _lid(1, 0).to_dict(), "allow_fallback": False})
        assert strict["route"]["lid"]["replica_idx"] == 0
        assert "error" in fr._handle_request({"method": "no_such_method"})
        b0.stop()
        b1.stop()
    finally:
        a.stop()


def test_tp_group_is_listed_whole_and_fails_as_one(fr):
    a = _client(fr, 0)
    gone = []
    a.on_event(EventType.ENDPOINT_DEREGISTERED, lambda e: gone.append(e.payload["lid"]["shard_idx"]))
    try:
        s0 = _client(fr, 1, 0, shard=0, group=2)
        assert wait_until(lambda: fr.route_manager.get_route(_lid(1, 0, 0)) is not None, 3)
        # one of two ranks: the instance is not serving yet
        assert a.get_stage_peers(1, refresh="always") == []
        s1 = _client(fr, 1, 0, shard=1, group=2)
        # complete: the instance serves through its shard 0
        assert wait_until(lambda: [(r.lid.shard_idx, r.group_size) for r in a.get_stage_peers(1, refresh="always")]
                          == [(0, 2)], 3)
        failed = a.report_failure(_lid(1, 0, 1), "rank died")
        assert sorted(failed) == sorted([_lid(1, 0, 0).to_key(), _lid(1, 0, 1).to_key()])
        assert wait_until(lambda: sorted(gone) == [0, 1], 3)
        assert a.get_stage_peers(1, refresh="always") == []
        s0.stop(deregister=False)
        s1.stop(deregister=False)
    finally:
        a.stop()


def test_one_rank_missing_its_lease_fails_the_group(fr):
    a = _client(fr, 0)
    gone = []
    a.on_event(EventType.ENDPOINT_DEREGISTERED, lambda e: gone.append((e.payload["lid"]["shard_idx"],
                                                                       e.payload.get("reason"))))
    try:
        s0 = _client(fr, 1, 0, shard=0, group=2)
        s1 = _client(fr, 1, 0, shard=1, group=2)
        assert wait_until(lambda: len(a.get_stage_peers(1, refresh="always")) == 1, 3)
        s1.kill()
        assert wait_until(lambda: sorted(s for s, _ in gone) == [0, 1], 3)
        assert {r for _, r in gone} == {"group_member_unhealthy"}
        s0.stop(deregister=False)
    finally:
        a.stop()

"""Directory server / client: registration, lookup, events, leases, failure reports."""
import threading
import time

import msgpack
import pytest
import zmq

from connex.directory import DirectoryClient, EndpointInfo, MembershipEvent, TransportCapability
from connex.directory_server import DirectoryServer
from tests.helpers import free_ports, wait_until


@pytest.fixture
def server():
    p, _ = free_ports(2)
    s = DirectoryServer(f"127.0.0.1:{p}", lease_s=0.5)
    s.start()
    yield s
    s.stop()


def client(server, stage, replica=0, addrs=None):
    c = DirectoryClient(server.bind_addr, "m", stage, replica_idx=replica, local_addresses=addrs or [])
    c.start()
    return c


def test_register_lookup_list(server):
    a = client(server, 1, 0, ["127.0.0.1:7000"])
    b = client(server, 1, 1, ["127.0.0.1:7001"])
    assert a.register() and b.register()
    q = client(server, 0)
    ep = q.lookup(("m", 1, 0, 1))
    assert ep is not None and ep.primary_address == "127.0.0.1:7001"
    assert [e.replica for e in q.list_stage(1)] == [0, 1]
    assert q.request_assignment(1, "forward") == ("127.0.0.1:7000", "m-1-0-0")
    assert q.list_stage(5) == []
    for c in (a, b, q):
        c.stop()


def test_epoch_bumps_and_events(server):
    q = client(server, 0)
    got = []
    q.subscribe_events(lambda ev, info: got.append((ev, info.lid, info.addresses)))
    assert q.start_event_listener()
    a = client(server, 1, 0, ["127.0.0.1:7000"])
    a.register()
    a.notify_migration(["127.0.0.1:7100"], target_epoch=5)
    a.deregister()
    assert wait_until(lambda: len(got) >= 3)
    assert [g[0] for g in got[:3]] == [MembershipEvent.JOIN, MembershipEvent.MIGRATE, MembershipEvent.LEAVE]
    assert got[1][2] == ["127.0.0.1:7100"]
    assert q.get_current_epoch() >= 3
    q.stop()
    a.stop()


def test_lease_expiry_and_reregister_on_heartbeat(server):
    q = client(server, 0)
    leaves = []
    q.subscribe_events(lambda ev, info: leaves.append(info.lid) if ev == MembershipEvent.LEAVE else None)
    q.start_event_listener()
    a = client(server, 1, 0, ["127.0.0.1:7000"])
    a.register()
    a.start_heartbeat(0.1)
    assert wait_until(lambda: ("m", 1, 0, 0) in server.members(), 2)
    # a peer reports it dead: evicted at once, then re-registers on its next heartbeat
    assert q.report_failure(("m", 1, 0, 0))
    assert wait_until(lambda: len(leaves) == 1, 2)
    assert wait_until(lambda: ("m", 1, 0, 0) in server.members(), 2)
    # stops heartbeating (process "died"): lease expires with reason "expired"
    a._hb_stop.set()
    assert wait_until(lambda: ("m", 1, 0, 0) not in server.members(), 3)
    q.stop()
    a.stop()


def test_members_without_heartbeat_are_kept(server):
    a = client(server, 1, 0, ["127.0.0.1:7000"])
    a.register()
    time.sleep(0.8)  # > lease, but never heartbeated
    assert ("m", 1, 0, 0) in server.members()
    a.stop()


def test_stale_reply_is_drained(server):
    c = client(server, 0)
    # a reply arriving after a timed-out call must not answer the next request
    c._control_socket.send(msgpack.packb({"type": "info"}, use_bin_type=True))
    time.sleep(0.1)
    r = c._control_call({"type": "list_stage", "model": "m", "stage": 3})
    assert r["status"] == "ok" and "endpoints" in r
    c.stop()


def test_endpoint_info_roundtrip():
    e = EndpointInfo(("m", 2, 1, 3), ["h:1"], [TransportCapability.ZEROMQ], epoch=4, metadata={"x": 1})
    e2 = EndpointInfo.from_dict(e.to_dict())
    assert e2.lid == ("m", 2, 1, 3) and e2.stage == 2 and e2.shard == 1 and e2.replica == 3
    assert e2.transport_caps == [TransportCapability.ZEROMQ] and e2.metadata == {"x": 1}


def test_malformed_and_unknown_requests(server):
    ctx = zmq.Context.instance()
    s = ctx.socket(zmq.DEALER)
    s.connect(f"tcp://{server.bind_addr}")
    s.send(msgpack.packb({"type": "nope"}))
    assert s.poll(2000)
    assert msgpack.unpackb(s.recv(), raw=False)["status"] == "error"
    s.send(b"\xc1garbage")
    assert s.poll(2000)
    assert msgpack.unpackb(s.recv(), raw=False)["status"] == "error"
    s.close(0)

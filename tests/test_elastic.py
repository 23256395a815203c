"""ElasticPeerSet over a real directory + ZeroMQ transport, and the mobility run."""
import threading
import time

import pytest

from connex.directory import DirectoryClient, EndpointInfo, MembershipEvent, TransportCapability
from connex.directory_server import DirectoryServer
from connex.elastic import ElasticPeerSet, ZmqTransport
from tests.helpers import free_ports, wait_until


class FakeTransport:
    """Records calls; connects can be slowed or failed."""

    def __init__(self, delay=0.0):
        self.delay = delay
        self.connected, self.closed, self.sent = [], [], []
        self.fail_send = set()
        self.lock = threading.Lock()

    def connect_sync(self, host, port):
        time.sleep(self.delay)
        ep = f"{host}:{port}#{len(self.connected)}"
        with self.lock:
            self.connected.append(ep)
        return ep

    def send_sync(self, ep, data, tag=0):
        if ep.split("#")[0] in self.fail_send:
            raise ConnectionError("peer gone")
        self.sent.append((ep, data))

    def close_endpoint(self, ep):
        with self.lock:
            self.closed.append(ep)


@pytest.fixture
def dirsrv():
    p, _ = free_ports(2)
    s = DirectoryServer(f"127.0.0.1:{p}", lease_s=5.0)
    s.start()
    yield s
    s.stop()


def _member(srv, rep, addr):
    c = DirectoryClient(srv.bind_addr, "m", 1, replica_idx=rep)
    c.start()
    assert c.register([addr])
    return c


def test_join_leave_migrate_failure(dirsrv):
    owner = DirectoryClient(dirsrv.bind_addr, "m", 0)
    owner.start()
    t = FakeTransport()
    peers = ElasticPeerSet(owner, t, stage_idx=1, drain_grace_s=0.05)
    a = _member(dirsrv, 0, "127.0.0.1:9000")
    peers.start()
    assert peers.wait_ready(1, 5)
    b = _member(dirsrv, 1, "127.0.0.1:9001")
    assert peers.wait_ready(2, 5)
    assert {peers.pick(), peers.pick()} == {("m", 1, 0, 0), ("m", 1, 0, 1)}
    # migrate: same LID, new address -> reconnect, old endpoint drained then closed
    old_ep = peers.endpoint(("m", 1, 0, 0))
    a.notify_migration(["127.0.0.1:9100"], 10)
    assert wait_until(lambda: peers.endpoint(("m", 1, 0, 0)) not in (None, old_ep), 5)
    assert wait_until(lambda: old_ep in t.closed, 5)
    # send failure -> mark_failed -> reported to the directory -> gone everywhere
    t.fail_send.add("127.0.0.1:9001")
    with pytest.raises(ConnectionError):
        peers.send(("m", 1, 0, 1), b"x")
    assert peers.peers() == [("m", 1, 0, 0)]
    assert wait_until(lambda: ("m", 1, 0, 1) not in dirsrv.members(), 5)
    assert peers.stats["failures"] == 1
    # leave
    a.deregister()
    assert wait_until(lambda: peers.peers() == [], 5)
    assert peers.pick() is None
    peers.stop()
    for c in (owner, a, b):
        c.stop()


def test_stale_connect_is_discarded(dirsrv):
    """A JOIN followed by LEAVE while the connect is still running must not
    leave a routable peer behind."""
    owner = DirectoryClient(dirsrv.bind_addr, "m", 0)
    owner.start()
    t = FakeTransport(delay=0.3)
    peers = ElasticPeerSet(owner, t, stage_idx=1, drain_grace_s=0.01)
    peers.start()
    a = _member(dirsrv, 0, "127.0.0.1:9200")
    time.sleep(0.1)
    a.deregister()
    time.sleep(0.6)
    assert peers.peers() == []
    assert wait_until(lambda: len(t.closed) == len(t.connected), 2)
    peers.stop()
    owner.stop()
    a.stop()


def test_poll_mode_without_event_stream(dirsrv):
    owner = DirectoryClient(dirsrv.bind_addr, "m", 0)
    owner.start()
    owner.start_event_listener = lambda *a, **k: False  # a directory that publishes nothing
    peers = ElasticPeerSet(owner, FakeTransport(), stage_idx=1, poll_s=0.05)
    peers.start()
    a = _member(dirsrv, 0, "127.0.0.1:9300")
    assert peers.wait_ready(1, 5)
    a.deregister()
    assert wait_until(lambda: peers.peers() == [], 5)
    peers.stop()
    owner.stop()
    a.stop()


def test_zmq_transport_roundtrip():
    rx = ZmqTransport()
    tx = ZmqTransport()
    ep = tx.connect_sync("127.0.0.1", rx.local_port)
    assert tx.connect_sync("127.0.0.1", rx.local_port) is ep  # cached by address
    tx.send_sync(ep, b"hello")
    assert rx.recv_sync(2000) == b"hello"
    tx.close_endpoint(ep)
    tx.stop_sync()
    rx.stop_sync()


def test_mobility_run_exactly_once_in_order():
    """1000 steps of 64 B (seed 0); replica 1 fails at 200, rejoins at 400;
    replica 0 migrates at 600 and leaves at 800."""
    from connex.examples.mobile_endpoints import check, run
    rep = run(steps=1000, seed=0)
    res = check(rep)
    assert res["exactly_once"] and res["in_order"] and res["live_only"] and res["payload_ok"], res
    # both replicas served traffic, replica 1 alone after replica 0 left
    assert set(res["per_replica"]) == {0, 1}
    tail = [d["replica"] for d in sorted(rep["deliveries"], key=lambda d: d["t"])[800:]]
    assert set(tail) == {1}
    mid = [d["replica"] for d in sorted(rep["deliveries"], key=lambda d: d["t"])[200:400]]
    assert set(mid) == {0}

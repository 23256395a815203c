"""Deterministic release of peer mappings on CPU (stand-ins for the driver
calls and for events): a forgotten peer's mappings are released only after
every fence of the streams that used them passed, never before; other
peers' mappings stay open; close() releases the rest; release errors do not
stop the reaper."""
import pytest

from connex_b200.parallel import peer
from connex_b200.parallel.peer import Graveyard, PeerHandle, PeerMapper


class Fence:
    def __init__(self):
        self.done = False

    def query(self):
        return self.done


@pytest.fixture
def fake_ipc(monkeypatch):
    opened, closed = {}, []

    def ipc_open(handle, device):
        base = 0x10000000 * (len(opened) + 1)
        opened[base] = handle
        return base

    monkeypatch.setattr(peer.ops, "ipc_open", ipc_open, raising=False)
    monkeypatch.setattr(peer.ops, "ipc_close", lambda base, device: closed.append(base), raising=False)
    return opened, closed


def _h(tag: bytes, pid: int, offset=0, nbytes=4096):
    return PeerHandle(tag * 64, offset, nbytes, 0, pid)


def test_graveyard_releases_only_after_fences_pass():
    g = Graveyard()
    released = []
    f1, f2 = Fence(), Fence()
    g.bury(f1.query, lambda: released.append("a"), 100, "a")
    g.bury(f2.query, lambda: released.append("b"), 50, "b")
    assert g.reap() == 2 and released == []
    f2.done = True
    assert g.reap() == 1 and released == ["b"] and g.released_bytes == 50
    f1.done = True
    assert g.drain(1.0) == 0 and released == ["b", "a"] and g.released == 2 and g.buried == 2


def test_graveyard_survives_a_failing_release():
    g = Graveyard()

    def boom():
        raise RuntimeError("context gone")
    g.bury(lambda: True, boom, 10, "x")
    g.bury(lambda: True, lambda: None, 20, "y")
    assert g.reap() == 0 and g.released == 2


def test_forgotten_peer_is_unmapped_after_its_streams_pass(fake_ipc):
    opened, closed = fake_ipc
    m = PeerMapper(0)
    a1 = m.open(_h(b"a", 101, offset=64), owner="peer-a")
    a2 = m.open(_h(b"a", 101, offset=128), owner="peer-a")      # same allocation: one mapping
    b1 = m.open(_h(b"b", 102), owner="peer-b")
    assert a2 - a1 == 64 and len(opened) == 2 and m.owners() == ["peer-a", "peer-b"]
    fence = Fence()                                              # a kernel still queued against peer-a
    assert m.forget("peer-a", fences=[fence]) == 1
    assert m.reap() == 1 and closed == []                        # not while the stream may touch it
    fence.done = True
    assert m.reap() == 0 and closed == [a1 - 64]
    assert m.owners() == ["peer-b"]
    # a new incarnation of peer-a maps afresh
    m.open(_h(b"a", 103), owner="peer-a")
    assert len(opened) == 3
    assert m.close(timeout_s=1.0) == 0 and sorted(closed) == sorted(opened)
    assert m.graveyard.released == 3


def test_close_keeps_a_mapping_that_is_still_in_use(fake_ipc):
    opened, closed = fake_ipc
    m = PeerMapper(0)
    m.open(_h(b"c", 104), owner="c")
    fence = Fence()
    m.forget("c", fences=[fence])
    assert m.close(timeout_s=0.05) == 1 and closed == []         # kept, not unmapped under a running copy
    fence.done = True
    assert m.reap() == 0 and len(closed) == 1


def test_handle_dict_round_trip_keeps_the_kind():
    h = PeerHandle(b"", 256, 4096, 1, 7, "vmm", {"sock": "s", "id": 3, "alloc_size": 2 << 20})
    g = PeerHandle.from_dict(h.to_dict())
    assert g == h and g.kind == "vmm" and g.key == ("vmm", "s", 3)
    legacy = PeerHandle.from_dict({"handle": b"x" * 64, "offset": 0, "nbytes": 1, "owner_device": 0, "owner_pid": 1})
    assert legacy.kind == "ipc" and legacy.key == ("ipc", b"x" * 64)

"""Native transfer engine over TCP on localhost (no GPU): the one-sided
transfer surface, GIL release, peer-death events and same-identity rejoin."""
import os
import threading
import time

import pytest

from connex_b200.engine import INVALID, PEER_FAILED, CxEngineTransport, Engine, url_hostport, url_identity


def _engine(stage, replica=0, port=0, **kw):
    return Engine("t", stage, 0, replica, listen_ip="127.0.0.1", port=port, **kw)


def _event(eng, kind, timeout_s=5.0):
    t = time.monotonic()
    while time.monotonic() - t < timeout_s:
        ev = eng.wait_event(100)
        if ev and ev["type"] == kind:
            return ev
    return None


def test_transfer_surface():
    a, b = _engine(0), _engine(1)
    try:
        assert url_identity(a.local_url) == ("t", 0, 0, 0) and a.port == int(url_hostport(a.local_url).split(":")[1])
        n = 1 << 20
        src, dst = a.allocate_managed_buffer(n), b.allocate_managed_buffer(n)
        data = os.urandom(n)
        a.write_bytes_to_buffer(src, data, n)
        assert b.transfer_sync_read(a.local_url, dst, src, n) == 0
        assert b.read_bytes_from_buffer(dst, n) == data
        # sub-range into memory registered by pointer
        buf = bytearray(4096)
        import ctypes
        cbuf = (ctypes.c_char * 4096).from_buffer(buf)
        ptr = ctypes.addressof(cbuf)
        assert b.register_memory(ptr, 4096) == 0
        assert b.transfer_sync_read(a.local_url, ptr, src + 100, 4096) == 0
        assert bytes(buf) == data[100:4196]
        assert b.unregister_memory(ptr) == 0
        del cbuf
        # unknown remote region: an error code, the link stays up
        assert b.transfer_sync_read(a.local_url, dst, 0x1000, 64) == INVALID
        assert b.transfer_sync_read(a.local_url, dst, src, 64) == 0
        # one-sided write + signal: data in place when the message arrives
        b.write_bytes_to_buffer(dst, b"x" * 64, 64)
        assert b.put_signal(a.local_url, dst, src, 64, b"sig").wait(5000) == 0
        peer, msg = a.recv_msg(5000)
        assert peer == ("t", 1, 0, 0) and msg == b"sig"
        assert a.read_bytes_from_buffer(src, 64) == b"x" * 64
        # async read, write
        h = b.get_async(a.local_url, dst, src + 64, 128)
        assert h.wait(5000) == 0 and b.read_bytes_from_buffer(dst, 128) == data[64:192]
        assert b.put_async(a.local_url, dst, src, 16).wait(5000) == 0
        assert b.transfer_sync_write(a.local_url, dst, src + 8, 8) == 0
        # messages by identity
        assert a.send_msg(("t", 1, 0, 0), b"hi")
        assert b.recv_msg(2000) == (("t", 0, 0, 0), b"hi")
        assert _event(b, "up")["peer"] == ("t", 0, 0, 0)
        assert _event(a, "joined")["peer"] == ("t", 1, 0, 0)
        a.free_managed_buffer(src, n)
        b.free_managed_buffer(dst, n)
        st = b.stats()
        assert st["inflight"] == 0 and st["regions"] == 0 and st["rma_ok"] >= 4 and st["rma_err"] == 1
    finally:
        a.close()
        b.close()


def test_blocking_calls_release_the_gil():
    a, b = _engine(0), _engine(1)
    try:
        n = 16 << 20
        src, dst = a.allocate_managed_buffer(n), b.allocate_managed_buffer(n)
        ticks = []
        stop = threading.Event()

        def spin():
            while not stop.is_set():
                ticks.append(time.monotonic())
                time.sleep(0.001)

        th = threading.Thread(target=spin)
        th.start()
        t0 = time.monotonic()
        for _ in range(10):
            assert b.transfer_sync_read(a.local_url, dst, src, n) == 0
        took = time.monotonic() - t0
        stop.set()
        th.join()
        assert len([x for x in ticks if x >= t0]) > took / 0.001 * 0.3
    finally:
        a.close()
        b.close()


def test_peer_failure_event_and_same_identity_rejoin():
    b = _engine(1)
    a = _engine(0)
    port, url = a.port, a.local_url
    try:
        src, dst = a.allocate_managed_buffer(4096), b.allocate_managed_buffer(4096)
        a.write_bytes_to_buffer(src, b"1" * 4096, 4096)
        assert b.transfer_sync_read(url, dst, src, 4096) == 0
        t0 = time.monotonic()
        a.close()
        ev = _event(b, "failed")
        assert ev is not None and ev["peer"] == ("t", 0, 0, 0)
        assert time.monotonic() - t0 < 1.0
        assert b.transfer_sync_read(url, dst, src, 4096, timeout_ms=1000) < 0
        a = _engine(0, port=port)
        assert a.local_url == url
        src = a.allocate_managed_buffer(4096)
        a.write_bytes_to_buffer(src, b"2" * 4096, 4096)
        for _ in range(50):
            if b.transfer_sync_read(url, dst, src, 4096) == 0:
                break
            time.sleep(0.05)
        assert b.read_bytes_from_buffer(dst, 4096) == b"2" * 4096
    finally:
        a.close()
        b.close()


def test_heartbeat_timeout_detects_silent_peer():
    """A peer that stops answering (no EOF) is failed by the heartbeat timeout."""
    b = Engine("t", 1, 0, 0, listen_ip="127.0.0.1", heartbeat_ms=50, heartbeat_timeout_ms=300)
    import socket
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    port = srv.getsockname()[1]

    def fake_peer():
        c, _ = srv.accept()
        hdr = c.recv(9)
        import struct
        n = struct.unpack("<Q", hdr[:8])[0]
        c.recv(n - 1)
        me = b"t|0|0|0"
        c.sendall(struct.pack("<Q", len(me) + 1) + bytes([2]) + me)
        time.sleep(3)  # then silence
        c.close()

    th = threading.Thread(target=fake_peer, daemon=True)
    th.start()
    try:
        assert b.connect(f"127.0.0.1:{port}")
        ev = _event(b, "failed", timeout_s=3)
        assert ev is not None and ev["reason"] == "heartbeat timeout"
    finally:
        b.close()
        srv.close()


def test_elastic_transport_adapter():
    a, b = _engine(0), _engine(1)
    try:
        t = CxEngineTransport(b)
        host, port = url_hostport(a.local_url).split(":")
        ep = t.connect_sync(host, int(port))
        t.send_sync(ep, b"payload")
        assert a.recv_msg(2000)[1] == b"payload"
        with pytest.raises(ConnectionError):
            t.connect_sync("127.0.0.1", 1)
    finally:
        a.close()
        b.close()

"""The transfer engine's device plane on a GPU: engine-allocated (VMM) and
registered (torch, legacy IPC) device regions read and written one-sided by
a peer process, put_chain's doorbell -> gate -> payload -> flag order with
its timeout and cancel, device memory refused to a peer on another machine,
and the graveyard: the memory of an exporter that was SIGKILLed between
steps stays alive while the importer maps it and is freed when the importer
releases its mappings (the peer processes are killed on the host; no GPU
fault is involved).  On a box with two or more GPUs the peer copies cross
NVLink; with one GPU both processes share it."""
import multiprocessing as mp
import os
import signal
import time

import pytest

pytestmark = pytest.mark.gpu

MiB = 1 << 20


def _exporter(q, cmd, port, device, big, env):
    os.environ.update(env)
    import torch

    from connex_b200.engine import Engine
    torch.cuda.set_device(device)
    eng = Engine("t", 0, 0, 0, listen_ip="127.0.0.1", port=port, heartbeat_timeout_ms=0)   # EOF finds deaths
    eng.set_device(device)
    q.put(("ready", eng.local_url))
    cmd.get(timeout=120)                                    # the importer measured its baseline
    n = 8 * MiB
    vmm = eng.allocate_device_buffer(big or n, device)
    pattern = bytes((i * 7 + 3) % 251 for i in range(n))
    eng.write_bytes_to_buffer(vmm, pattern, n)
    t = torch.arange((1 << 30) // 4 if big else n // 4, dtype=torch.int32, device=device)   # 1 GiB / 8 MiB
    assert eng.register_memory(t.data_ptr(), t.numel() * 4) == 0
    host = eng.allocate_managed_buffer(n)
    eng.write_bytes_to_buffer(host, pattern[::-1], n)
    q.put(("regions", vmm, t.data_ptr(), host, eng.region_kind(vmm), eng.region_kind(t.data_ptr()),
           eng.region_kind(host)))
    cmd.get(timeout=300)                                    # until told to exit (or killed)
    eng.close()


class _Peer:
    def __init__(self, device, port=0, big=0, env=None):
        ctx = mp.get_context("spawn")
        self.q, self.cmd = ctx.Queue(), ctx.Queue()
        self.p = ctx.Process(target=_exporter, args=(self.q, self.cmd, port, device, big, env or {}), daemon=True)
        self.p.start()
        kind, self.url = self.q.get(timeout=180)

    def regions(self):
        self.cmd.put("go")
        _, self.vmm, self.tensor, self.host, *kinds = self.q.get(timeout=180)
        return kinds

    def stop(self):
        if self.p.is_alive():
            self.cmd.put("exit")
            self.p.join(30)
        if self.p.is_alive():
            self.p.kill()


def _devices():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    n = torch.cuda.device_count()
    return (0, 1) if n >= 2 else (0, 0)


def _importer(device, **kw):
    from connex_b200.engine import Engine
    eng = Engine("t", 1, 0, 0, listen_ip="127.0.0.1", **kw)
    eng.set_device(device)
    return eng


def test_device_regions_one_sided_and_put_chain():
    from connex_b200.engine import CANCELLED, INVALID, TIMEOUT, device_plane
    assert device_plane()[0], device_plane()[1]
    dev_a, dev_b = _devices()
    a = _Peer(dev_a)
    b = _importer(dev_b)
    try:
        assert a.regions() == ["vmm", "ipc", "host"]
        n = 8 * MiB
        pattern = bytes((i * 7 + 3) % 251 for i in range(n))
        dst = b.allocate_device_buffer(n, dev_b)
        assert b.region_kind(dst) == "vmm"
        # device <- peer device (VMM export), then host <- peer device (torch tensor, IPC export)
        assert b.transfer_sync_read(a.url, dst, a.vmm, n) == 0
        assert b.read_bytes_from_buffer(dst, n) == pattern
        hbuf = b.allocate_managed_buffer(n)
        assert b.transfer_sync_read(a.url, hbuf, a.tensor, 4096) == 0
        import struct
        assert struct.unpack("<4i", b.read_bytes_from_buffer(hbuf, 16)) == (0, 1, 2, 3)
        # peer device <- local device, read back; peer host <- local device (bounce)
        b.write_bytes_to_buffer(dst, b"\x5a" * 4096, 4096)
        assert b.transfer_sync_write(a.url, dst, a.vmm + 4096, 4096) == 0
        assert b.transfer_sync_read(a.url, hbuf, a.vmm, 3 * 4096) == 0
        got = b.read_bytes_from_buffer(hbuf, 3 * 4096)
        assert got[:4096] == pattern[:4096] and got[4096:8192] == b"\x5a" * 4096
        assert b.transfer_sync_write(a.url, dst, a.host, 4096) == 0
        assert b.transfer_sync_read(a.url, dst + 4096, a.host, 4096) == 0
        assert b.read_bytes_from_buffer(dst + 4096, 4096) == b"\x5a" * 4096
        # async, and an unknown range (past the allocation's registered size)
        assert b.get_async(a.url, dst, a.vmm + 64, 1024).wait(5000) == 0
        assert b.put_async(a.url, dst, a.vmm + 8192, 1024).wait(5000) == 0
        assert b.transfer_sync_read(a.url, dst, a.vmm + n, 64) == INVALID
        # put_chain: waits for the doorbell, then payload, then the flag
        ring, flag, gate = a.vmm + 1 * MiB, a.vmm + 2 * MiB, a.vmm + 2 * MiB + 64
        b.write_bytes_to_buffer(hbuf, b"\0" * 16, 16)            # bell = 0, cancel = 0
        b.transfer_sync_write(a.url, hbuf, gate, 4)              # gate word = 0
        b.write_bytes_to_buffer(dst, b"\xc3" * 65536, 65536)
        h = b.put_chain(a.url, hbuf, 1, gate, 0, dst, ring, 65536, flag, 7, queue=1, timeout_ms=5000)
        time.sleep(0.05)
        assert not h.done()                                     # no doorbell yet
        b.write_bytes_to_buffer(hbuf, struct.pack("<I", 1), 4)
        assert h.wait(5000) == 0
        assert b.transfer_sync_read(a.url, hbuf + 64, flag, 4) == 0
        assert struct.unpack("<I", b.read_bytes_from_buffer(hbuf + 64, 4))[0] == 7
        assert b.transfer_sync_read(a.url, hbuf + 128, ring, 65536) == 0
        assert b.read_bytes_from_buffer(hbuf + 128, 65536) == b"\xc3" * 65536
        # the gate is not open: bounded wait; a cancel word ends an armed chain
        assert b.put_chain(a.url, 0, 0, gate, 5, dst, ring, 64, flag, 8, timeout_ms=200).wait(5000) == TIMEOUT
        h = b.put_chain(a.url, hbuf, 9, 0, 0, dst, ring, 64, flag, 9, queue=2, cancel=hbuf + 4, arm_timeout_ms=5000)
        b.write_bytes_to_buffer(hbuf + 4, struct.pack("<I", 1), 4)
        assert h.wait(5000) == CANCELLED
        st = b.stats()
        assert st["imports"] >= 2 and st["dev_copies"] >= 6 and st["chains_ok"] == 1 and st["chains_err"] == 2
    finally:
        a.stop()
        b.close()


def test_device_memory_is_refused_to_another_machine():
    from connex_b200.engine import INVALID
    dev_a, dev_b = _devices()
    a = _Peer(dev_a, env={"CONNEX_ENGINE_HOST_ID": "another-machine"})
    b = _importer(dev_b)
    try:
        a.regions()
        hbuf = b.allocate_managed_buffer(4096)
        assert b.transfer_sync_read(a.url, hbuf, a.vmm, 4096) == INVALID      # no host memcpy of a device address
        assert b.transfer_sync_read(a.url, hbuf, a.tensor, 4096) == INVALID
        assert b.transfer_sync_read(a.url, hbuf, a.host, 4096) == 0           # host memory still travels
    finally:
        a.stop()
        b.close()


def test_dead_exporter_memory_is_released_by_the_importer():
    from connex_b200.engine import device_memory_info
    dev_a, dev_b = _devices()
    big = 4 << 30
    a = _Peer(dev_a, big=big)
    b = _importer(dev_b, heartbeat_ms=60000, heartbeat_timeout_ms=0)     # only the explicit reap releases
    try:
        free0 = device_memory_info(dev_a)[0]
        a.regions()
        hbuf = b.allocate_managed_buffer(4096)
        assert b.transfer_sync_read(a.url, hbuf, a.vmm + big - 4096, 4096) == 0   # maps the 4 GiB allocation
        assert b.transfer_sync_read(a.url, hbuf, a.tensor, 4096) == 0            # and the 1 GiB tensor's block
        st = b.stats()
        assert st["imports"] == 2 and st["import_bytes"] >= big
        port = int(a.url.split("#")[0].rsplit(":", 1)[1])
        os.kill(a.p.pid, signal.SIGKILL)                                   # between steps: nothing in flight
        a.p.join(30)
        end = time.monotonic() + 10
        ev = None
        while time.monotonic() < end and not (ev and ev["type"] == "failed"):
            ev = b.wait_event(200)
        assert ev and ev["type"] == "failed"
        time.sleep(1.0)                                                    # the exporter's context is gone
        free_dead = device_memory_info(dev_a)[0]
        assert free_dead < free0 - (big * 3) // 4                          # still alive: the importer maps it
        assert b.stats()["graveyard"] == 2
        assert b.reap(5000) == 0
        end = time.monotonic() + 10
        while time.monotonic() < end and device_memory_info(dev_a)[0] < free_dead + (big * 3) // 4:
            time.sleep(0.1)
        assert device_memory_info(dev_a)[0] >= free_dead + (big * 3) // 4   # freed with the last mapping
        st = b.stats()
        assert st["released"] == 2 and st["released_bytes"] >= big + (1 << 30) and st["imports"] == 0
        # the peer comes back at the same URL: its new regions resolve on the new link
        a2 = _Peer(dev_a, port=port)
        try:
            a2.regions()
            assert b.transfer_sync_read(a2.url, hbuf, a2.vmm, 4096) == 0
        finally:
            a2.stop()
    finally:
        a.stop()
        b.close()


def _tensor_exporter(q, cmd, device, nbytes):
    import torch

    from connex_b200.parallel.peer import export_tensor, shared_empty
    torch.cuda.set_device(device)
    q.put(("ready", None))
    cmd.get(timeout=120)
    t = shared_empty((nbytes,), torch.uint8, device)
    t.copy_(torch.arange(nbytes, device=device, dtype=torch.int64).remainder_(251).to(torch.uint8))
    torch.cuda.synchronize(device)
    q.put(("regions", export_tensor(t[4096:]).to_dict(), None, None))
    cmd.get(timeout=300)


def test_shared_tensor_of_a_dead_peer_is_released_by_the_mapper():
    import torch

    from connex_b200 import ops
    from connex_b200.parallel.peer import PeerHandle, PeerMapper
    dev_a, dev_b = _devices()
    nbytes = 2 << 30
    ctx = mp.get_context("spawn")
    q, cmd = ctx.Queue(), ctx.Queue()
    p = ctx.Process(target=_tensor_exporter, args=(q, cmd, dev_a, nbytes), daemon=True)
    p.start()
    try:
        q.get(timeout=180)
        free0 = torch.cuda.mem_get_info(dev_a)[0]
        cmd.put("go")
        _, hd, _, _ = q.get(timeout=180)
        h = PeerHandle.from_dict(hd)
        assert h.kind == "vmm" and h.offset == 4096
        mapper = PeerMapper(dev_b)
        addr = mapper.open(h, owner="a")
        dst = torch.zeros(8192, dtype=torch.uint8, device=dev_b)
        segs = torch.tensor([[addr, dst.data_ptr(), 8192]], dtype=torch.int64, device=dev_b)
        with torch.cuda.device(dev_b):
            ops.copy_segments(segs, 8192)
        torch.cuda.synchronize(dev_b)
        want = (torch.arange(4096, 4096 + 8192) % 251).to(torch.uint8)
        assert torch.equal(dst.cpu(), want)
        os.kill(p.pid, signal.SIGKILL)                       # the owner dies between steps
        p.join(30)
        time.sleep(1.0)
        free_dead = torch.cuda.mem_get_info(dev_a)[0]
        assert free_dead < free0 - nbytes // 2                # kept alive by this process's mapping
        assert mapper.forget("a", streams=[torch.cuda.current_stream(dev_b)]) == 1
        assert mapper.graveyard.drain(5.0) == 0
        end = time.monotonic() + 10
        while time.monotonic() < end and torch.cuda.mem_get_info(dev_a)[0] < free_dead + nbytes // 2:
            time.sleep(0.1)
        assert torch.cuda.mem_get_info(dev_a)[0] >= free_dead + nbytes // 2
        assert mapper.graveyard.released_bytes >= nbytes
    finally:
        if p.is_alive():
            p.kill()

"""Race regressions and threading stress of the PP endpoint and the native
engine, on CPU over real sockets.

* a late duplicate reply of an answered step must never be taken for the
  next step (wrong tokens), even when the next step's waiter is already
  blocked when the duplicate arrives;
* a reply that arrives before anyone waits for it must be returned at once
  (not treated as lost, no timeout);
* a duplicate step reaching a later stage is answered from its reply cache,
  never computed twice;
* many threads sending steps and control messages through one endpoint at
  once get exactly their own replies;
* many threads using one native engine at once (one-sided reads and writes
  into their own regions, messages) see their own bytes and no error.

Each stress test arms ``faulthandler`` so a hang dumps every thread's stack
instead of stalling the suite.  Behavioural parity: the reference's race
regressions in ``tests/test_pp_core.py:507-559``.
"""
import faulthandler
import os
import random
import sys
import threading
import time

import pytest
import torch

from connex.pp.endpoint import PipelineEndpoint
from connex.pp.routing import StaticMembership
from tests.helpers import wait_until


@pytest.fixture
def watchdog():
    faulthandler.dump_traceback_later(90, exit=False, file=sys.stderr)
    yield
    faulthandler.cancel_dump_traceback_later()


def _pair(timeout=10.0, k=1):
    mem = StaticMembership(0, 0)
    s0 = PipelineEndpoint("m", 0, 2, 0, membership=mem, recv_timeout_s=timeout, k=k)
    s1 = PipelineEndpoint("m", 1, 2, 0, membership=mem, recv_timeout_s=timeout, k=k)
    mem.add(0, 0, s0.address)
    mem.add(1, 0, s1.address)
    return s0, s1


def test_late_duplicate_reply_is_never_taken_for_the_next_step(watchdog):
    s0, s1 = _pair()
    try:
        c1 = s0.new_step_id()
        s0.send_step({"h": torch.zeros(1)}, c1)
        td, ctx = s1.recv_forward(5)
        s1.send_reply({"h": td["h"] + 1}, ctx)
        s1.send_reply({"h": td["h"] + 1}, ctx)               # a late duplicate of the same answer
        assert s0.recv_step(c1, 5)["h"].item() == 1.0
        got = {}
        c2 = s0.new_step_id()
        th = threading.Thread(target=lambda: got.setdefault("r", s0.recv_step(c2, 5)))
        th.start()                                          # the next step's waiter is already blocked
        time.sleep(0.05)
        s1._send_reply_now({"h": torch.full((1,), 99.0)}, c1, s0.address)   # another stale copy, mid-wait
        s0.send_step({"h": torch.full((1,), 10.0)}, c2)
        td, ctx = s1.recv_forward(5)
        s1.send_reply({"h": td["h"] + 1}, ctx)
        th.join(5)
        assert got["r"]["h"].item() == 11.0
        assert wait_until(lambda: s0.stats["late_replies"] >= 1, 2)      # the mid-wait copy, at least
    finally:
        s0.close()
        s1.close()


def test_a_reply_that_arrives_before_the_waiter_is_returned_at_once(watchdog):
    s0, s1 = _pair()
    try:
        c = s0.new_step_id()
        s0.send_step({"h": torch.zeros(1)}, c)
        td, ctx = s1.recv_forward(5)
        s1.send_reply({"h": td["h"] + 1}, ctx)
        assert wait_until(lambda: c in s0._done, 3)          # delivered, nobody waiting yet
        t = time.monotonic()
        assert s0.recv_step(c, 5)["h"].item() == 1.0
        assert time.monotonic() - t < 0.3
    finally:
        s0.close()
        s1.close()


def test_a_duplicate_step_is_answered_from_the_reply_cache(watchdog):
    s0, s1 = _pair()
    computed = []
    try:
        c = s0.new_step_id()
        s0.send_step({"h": torch.zeros(1)}, c)
        td, ctx = s1.recv_forward(5)
        computed.append(ctx[0])
        s1.send_reply({"h": td["h"] + 5}, ctx)
        assert s0.recv_step(c, 5)["h"].item() == 5.0
        c_again = c
        with s0._cv:
            s0._outstanding.add(c_again)                    # the same step re-sent (e.g. after a timeout)
        s0.send_step({"h": torch.zeros(1)}, c_again)
        assert s0.recv_step(c_again, 5)["h"].item() == 5.0
        assert s1.recv_forward(0.2) == (None, None)         # never reached the worker a second time
        assert s1.stats["dedup_replies"] == 1 and computed == [c]
    finally:
        s0.close()
        s1.close()


def test_concurrent_steps_and_control_messages_get_their_own_replies(watchdog):
    s0, s1 = _pair(timeout=20.0, k=8)                     # eight steps in flight: one per sender
    stop = threading.Event()
    pongs = []
    s0.control_handlers.append(lambda m: pongs.append(m) if m.get("kind") == "PONG" else None)
    s1.control_handlers.append(lambda m: s1.send_control(m["from"], {"kind": "PONG", "n": m["n"]})
                               if m.get("kind") == "PING" else None)

    def stage1():
        while not stop.is_set():
            td, ctx = s1.recv_forward(0.1)
            if td is not None:
                if random.random() < 0.2:
                    time.sleep(random.random() * 0.002)
                s1.send_reply({"h": td["h"] * 2 + 1, "tag": td["tag"]}, ctx)

    workers = [threading.Thread(target=stage1, daemon=True) for _ in range(2)]
    for w in workers:
        w.start()
    errors = []

    def sender(k):
        rng = random.Random(k)
        for i in range(60):
            c = s0.new_step_id()
            v = float(k * 1000 + i)
            s0.send_step({"h": torch.full((3,), v), "tag": f"{k}/{i}"}, c)
            if rng.random() < 0.3:
                s0.send_control(s1.address, {"kind": "PING", "n": k * 1000 + i})
            r = s0.recv_step(c, 10)
            if r is None or r["tag"] != f"{k}/{i}" or r["h"][0].item() != v * 2 + 1:
                errors.append((k, i, None if r is None else (r["tag"], r["h"][0].item())))

    try:
        threads = [threading.Thread(target=sender, args=(k,)) for k in range(8)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(60)
        assert not any(t.is_alive() for t in threads)
        assert errors == []
        assert wait_until(lambda: len(pongs) == s0.stats.get("control_pong", 0) and len(pongs) > 0, 5)
        assert s1.stats["stale_dropped"] == 0 and not s0._outstanding
    finally:
        stop.set()
        s0.close()
        s1.close()


def test_native_engine_under_concurrent_use(watchdog):
    pytest.importorskip("connex_b200._cxengine")
    from connex_b200.engine import Engine
    a = Engine("t", 0, 0, 0, listen_ip="127.0.0.1")
    b = Engine("t", 1, 0, 0, listen_ip="127.0.0.1")
    n, threads_n = 1 << 16, 8
    errors = []
    try:
        regions = [a.allocate_managed_buffer(n) for _ in range(threads_n)]
        locals_ = [b.allocate_managed_buffer(n) for _ in range(threads_n)]

        def worker(k):
            rng = random.Random(k)
            for it in range(40):
                data = os.urandom(n)
                b.write_bytes_to_buffer(locals_[k], data, n)
                if b.transfer_sync_write(a.local_url, locals_[k], regions[k], n) != 0:
                    errors.append(("write", k, it))
                    continue
                b.write_bytes_to_buffer(locals_[k], b"\0" * n, n)
                off = rng.randrange(0, n - 4096) & ~15
                if b.transfer_sync_read(a.local_url, locals_[k] + off, regions[k] + off, 4096) != 0:
                    errors.append(("read", k, it))
                    continue
                if b.read_bytes_from_buffer(locals_[k] + off, 4096) != data[off:off + 4096]:
                    errors.append(("bytes", k, it))
                h = b.get_async(a.local_url, locals_[k], regions[k], 256)
                if h.wait(5000) != 0:
                    errors.append(("async", k, it))
                if not b.send_msg(a.local_url, f"{k}:{it}".encode()):
                    errors.append(("msg", k, it))

        threads = [threading.Thread(target=worker, args=(k,)) for k in range(threads_n)]
        for t in threads:
            t.start()
        got = []
        end = time.monotonic() + 60
        while len(got) < threads_n * 40 and time.monotonic() < end:
            m = a.recv_msg(200)
            if m is not None:
                got.append(m[1])
        for t in threads:
            t.join(60)
        assert errors == []
        assert sorted(got) == sorted(f"{k}:{i}".encode() for k in range(threads_n) for i in range(40))
        st = b.stats()
        assert st["inflight"] == 0 and st["rma_err"] == 0 and st["failures"] == 0
    finally:
        a.close()
        b.close()

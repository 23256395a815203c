"""RL weight-sync edge cases on CPU: a copy overwritten while it is read is
reported stale to its readers, a copy being retired gets no new readers, a
subscriber re-reads when its source was overwritten mid-read, a single-buffer
publisher retires the version it overwrites, and a failed pull exposes no
previous manifest."""
import threading
import time

import pytest
import torch

from connex.rl.registry import PUBLISHER, WeightRegistry
from connex.rl.sync import WeightPublisher, WeightSubscriber
from connex.rl.transport import LocalTransport


def _weights(v: float):
    return [("a", torch.full((64, 32), v)), ("b", torch.arange(100, dtype=torch.float32) + v)]


def test_copy_overwritten_during_a_read_is_reported_stale():
    reg = WeightRegistry()
    reg.publish(version=1, manifest={}, url="pub", addr=0)
    src = reg.assign(version=1, member="r1")
    assert src["member"] == PUBLISHER
    assert reg.wait_idle(version=1, timeout=0.05)["ok"] is False       # reader still on it: overwritten anyway
    assert reg.release(version=1, source=PUBLISHER, member="r1") == {"ok": True, "stale": True}
    assert reg.release(version=1, source=PUBLISHER, member="r1") == {"ok": True}   # said once


def test_a_retiring_copy_gets_no_new_readers():
    reg = WeightRegistry()
    reg.publish(version=1, manifest={}, url="pub", addr=0)
    assert reg.assign(version=1, member="r1")["member"] == PUBLISHER
    t = threading.Thread(target=reg.wait_idle, kwargs={"version": 1, "timeout": 1.0, "retire": True})
    t.start()
    time.sleep(0.05)
    assert reg.assign(version=1, member="r2") is None                   # retiring: no new reader
    reg.release(version=1, source=PUBLISHER, member="r1")
    t.join(2)
    assert PUBLISHER not in reg.holders[1]


def test_subscriber_rereads_when_its_source_was_overwritten():
    reg = WeightRegistry()
    pt = LocalTransport("pub-rr")
    pub = WeightPublisher(reg, pt)
    pub.publish(_weights(1.0))
    st = LocalTransport("sub-rr")
    sub = WeightSubscriber(reg, st, "s1", heartbeat_s=0, chunk_bytes=1024)
    reads = {"n": 0}
    real = st.read_window

    def read_window(url, ops, dst, window=16, timeout_ms=None):
        reads["n"] += 1
        out = real(url, ops, dst, window, timeout_ms)
        if reads["n"] == 1:                                   # the publisher overwrote its copy meanwhile
            with reg.cv:
                reg.invalidate(1, PUBLISHER)
        return out
    st.read_window = read_window
    m = sub.pull()
    assert reads["n"] == 2 and m.version == 1
    got = dict(sub.tensors())
    assert torch.equal(got["a"], torch.full((64, 32), 1.0))


def test_single_buffer_publisher_retires_the_version_it_overwrites():
    reg = WeightRegistry()
    pub = WeightPublisher(reg, LocalTransport("pub-1buf"), buffers=1, idle_timeout=0.2)
    pub.publish(_weights(1.0))
    assert PUBLISHER in reg.holders[1]
    pub.publish(_weights(2.0))
    assert PUBLISHER not in reg.holders.get(1, {}) and PUBLISHER in reg.holders[2]


def test_failed_pull_exposes_no_previous_manifest():
    reg = WeightRegistry()
    pt = LocalTransport("pub-fail")
    pub = WeightPublisher(reg, pt)
    pub.publish(_weights(1.0))
    sub = WeightSubscriber(reg, LocalTransport("sub-fail"), "s2", heartbeat_s=0, max_source_failures=1)
    sub.pull()
    sub.commit(1)
    pub.publish(_weights(2.0))
    pt.kill()                                                  # the only source of v2 is gone
    with pytest.raises(Exception):
        sub.pull()
    assert sub.manifest is None
    with pytest.raises(Exception):
        dict(sub.tensors())

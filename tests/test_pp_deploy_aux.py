"""Deployment pieces of external PP without torch or vLLM: HMAC-sealed
control frames, the port layout and its CLI, and CONNEX_PP_TRACE step stamps
merged into one timeline (the stamps come from a real Stage0Link /
StageWorker chain)."""
import subprocess
import sys
import threading

import pytest

from connex.adapters.vllm.pp import auth, ports


def test_frames_verify_and_tampering_is_rejected(tmp_path):
    key = auth.load_secret({"CONNEX_PP_SECRET": "0123456789abcdef-secret"})
    fa = auth.FrameAuth(key)
    frame = fa.seal(b"payload")
    assert frame[:4] == b"CXA1" and len(frame) == 4 + 16 + 7 and bytes(fa.open(frame)) == b"payload"
    bad = bytearray(frame)
    bad[-1] ^= 1
    assert fa.open(bytes(bad)) is None and fa.open(b"xx") is None and fa.rejected == 2
    assert auth.FrameAuth(auth.load_secret({"CONNEX_PP_SECRET": "another-secret-of-16"})).open(frame) is None
    (tmp_path / "s").write_bytes(b"  file-secret-0123456789 \n")
    assert auth.load_secret({"CONNEX_PP_SECRET_FILE": str(tmp_path / "s")}) == b"file-secret-0123456789"
    assert auth.load_secret({"CONNEX_PP_AUTH": "off"}) is None
    off = auth.FrameAuth(None)
    assert off.seal(b"x") == b"x" and bytes(off.open(b"x")) == b"x"
    with pytest.raises(auth.AuthError):
        auth.load_secret({})
    with pytest.raises(auth.AuthError):
        auth.load_secret({"CONNEX_PP_SECRET": "short"})


def test_port_layout_never_collides(monkeypatch):
    monkeypatch.delenv("CONNEX_PP_PORT_BASE", raising=False)
    assert ports.control_port(1, 0) == 48000 and ports.data_port(1, 2, 3) == 48036
    seen = set()
    for s in range(3):
        for r in range(ports.MAX_REPLICAS):
            block = [ports.control_port(s, r)] + [ports.data_port(s, r, t) for t in range(ports.MAX_TP)]
            assert not seen & set(block)
            seen |= set(block)
    assert ports.rank_port(0, 3) == 0 and ports.rank_port(5000, 3) == 5003
    for bad in (lambda: ports.control_port(0, 62), lambda: ports.data_port(0, 0, 15), lambda: ports.control_port(64, 0)):
        with pytest.raises(ValueError):
            bad()
    out = subprocess.run([sys.executable, "-m", "connex.adapters.vllm.pp.ports", "data", "2", "1", "4"],
                         capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == str(47000 + 2000 + 16 + 5)


def test_step_trace_merges_a_chain_timeline(tmp_path, monkeypatch):
    import torch
    from connex.pp import steptrace
    from connex.pp.link import Stage0Link, StageWorker
    from connex.pp.testing import fake_chain
    monkeypatch.setattr(steptrace, "ON", True)
    monkeypatch.setattr(steptrace, "_file", None)
    monkeypatch.setenv("CONNEX_PP_TRACE_DIR", str(tmp_path))
    links = fake_chain(3)

    class H:
        def kv_held(self, r):
            return 0

        def release(self, r):
            pass

    stop = threading.Event()
    workers = [StageWorker(l, H(), lambda td, miss: {"x": td["x"] + 1}) for l in links[1:]]

    def serve(w):
        while not stop.is_set():
            w.serve_one()
    ts = [threading.Thread(target=serve, args=(w,), daemon=True) for w in workers]
    for t in ts:
        t.start()
    s0 = Stage0Link(links[0], H(), recv_timeout_s=1.0)
    for i in range(4):
        assert s0.step({"x": torch.tensor([float(i)])})["x"].item() == i + 2
    stop.set()
    for t in ts:
        t.join(2)
    steptrace.flush()
    files = [str(p) for p in tmp_path.glob("cxtrace-*.txt")]
    tl = steptrace.timeline(steptrace.load(files))
    assert len(tl) == 4
    for tags in tl.values():
        order = [t for t, _ in sorted(tags.items(), key=lambda kv: kv[1])]
        assert order == ["s0_send", "s1_recv", "s1_send", "s2_recv", "s2_send", "s0_reply"]
    out = subprocess.run([sys.executable, "-m", "connex.adapters.vllm.pp.trace", *files], capture_output=True,
                         text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.splitlines()[-1].startswith("median s0_send=+0.0")


def test_nvtx_ranges_only_when_enabled(monkeypatch):
    import torch
    from connex_b200.utils import nvtx
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: calls.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    monkeypatch.setattr(nvtx, "ON", False)
    with nvtx.nvtx_range("off"):
        pass
    assert calls == []
    monkeypatch.setattr(nvtx, "ON", True)
    with pytest.raises(ValueError):
        with nvtx.nvtx_range("ep dispatch"):
            raise ValueError("the range still closes")
    assert calls == [("push", "ep dispatch"), ("pop",)]

"""The serving pipeline through its CLIs on CPU (stand-in stages, no GPU): a
directory, stage 0 (`python -m connex_b200.serve --rule --num-stages 2`) and
two replicas of stage 1 (`python -m connex_b200.serve.stage --rule`), each
its own process.  The replica serving a stream is SIGKILLed mid-stream;
stage 0 fails over to the other replica, which lacks the request's KV, so
the rows are prefilled again there -- and the stream completes with exactly
the uninterrupted output."""
import os
import signal
import socket
import subprocess
import sys
import time
import urllib.request

from connex.serving.fake_backend import reference
from tests.test_serving import _run, _stream, _text


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _up(url, timeout=60):
    end = time.monotonic() + timeout
    while time.monotonic() < end:
        try:
            if urllib.request.urlopen(url + "/health", timeout=1).status == 200:
                return True
        except OSError:
            time.sleep(0.2)
    return False


def test_pipeline_cli_failover_keeps_the_stream_exact(tmp_path):
    env = dict(os.environ, PYTHONPATH=os.getcwd())
    dport, hport = _port(), _port()
    d = f"127.0.0.1:{dport}"
    procs = {}

    def start(name, args):
        f = open(tmp_path / f"{name}.log", "w")
        procs[name] = (subprocess.Popen([sys.executable, "-m"] + args, env=env, stdout=f, stderr=subprocess.STDOUT), f)

    def stage(r):
        start(f"s1r{r}", ["connex_b200.serve.stage", "--rule", "--rule-delay-ms", "25", "--num-stages", "2",
                          "--stage", "1", "--replica", str(r), "--directory", d, "--recv-timeout-s", "2"])
    try:
        start("dir", ["connex.directory_server", "--bind", d, "--lease", "1.0"])
        time.sleep(1.0)
        stage(0)
        time.sleep(1.5)
        start("s0", ["connex_b200.serve", "--rule", "--num-stages", "2", "--directory", d, "--port", str(hport),
                     "--host", "127.0.0.1", "--recv-timeout-s", "2"])
        url = f"http://127.0.0.1:{hport}"
        assert _up(url), (tmp_path / "s0.log").read_text()[-2000:]
        req = urllib.request.Request(url + "/v1/completions", data=b'{"prompt": "t5 t6", "max_tokens": 4}',
                                     headers={"Content-Type": "application/json"})
        assert b"t" in urllib.request.urlopen(req, timeout=30).read()          # served by replica 0
        stage(1)
        from connex.directory import DirectoryClient
        probe = DirectoryClient(d, "connex-b200", 9, replica_idx=99)
        probe.start()
        try:
            end = time.monotonic() + 60
            while len(probe.list_stage(1)) < 2:                                 # replica 1 registered
                assert time.monotonic() < end, (tmp_path / "s1r1.log").read_text()[-2000:]
                time.sleep(0.2)
        finally:
            probe.stop()
        time.sleep(1.0)                                                         # stage 0 hears of it and warms it

        async def stream_and_kill():
            import asyncio
            task = asyncio.ensure_future(_stream(url, "/v1/completions", {"prompt": "t7 t8", "max_tokens": 60}))
            await asyncio.sleep(0.6)
            procs["s1r0"][0].send_signal(signal.SIGKILL)                        # dies between or during steps
            return await task
        chunks, done = _run(stream_and_kill())
        assert done and _text(chunks) == reference("t7 t8", 60)[1]
        log1 = (tmp_path / "s1r1.log").read_text()
        assert "no KV here" in log1, log1[-2000:]                               # re-prefilled on replica 1
        log0 = (tmp_path / "s0.log").read_text()
        assert "transport:" in log0, log0[-3000:]                               # the engine's peer event moved it
    finally:
        for p, f in procs.values():
            if p.poll() is None:
                p.send_signal(signal.SIGTERM)
        for p, f in procs.values():
            try:
                p.wait(10)
            except subprocess.TimeoutExpired:
                p.kill()
            f.close()

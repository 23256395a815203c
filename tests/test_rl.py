"""RL weight sync on CPU: arena manifest, registry (in-process and over
HTTP), tree fan-out, source failover, double buffering, TTL expiry, the
rollout pool's one-version-per-request invariant, and the engine glue."""
import asyncio
import json
import threading
import time

import pytest
import torch

from connex.rl import (LocalTransport, RegistryClient, RegistryServer, RolloutPool, TransferError,
                       WeightManifest, WeightPublisher, WeightRegistry, WeightSubscriber, pack_into, unpack)
from connex.rl.fake import FakeInstance, expected, weights_for
from connex.rl.registry import PUBLISHER


def _named():
    return [("a", torch.arange(10, dtype=torch.float32)), ("b", torch.ones(3, 5, dtype=torch.bfloat16)),
            ("c", torch.tensor([7], dtype=torch.int64))]


def test_manifest_pack_unpack_roundtrip():
    named = _named()
    m = WeightManifest.build(3, named)
    assert all(e.offset % 256 == 0 for e in m.entries) and m.total % 256 == 0
    arena = torch.zeros(m.total, dtype=torch.uint8)
    pack_into(arena, m, named)
    m2 = WeightManifest.from_dict(json.loads(json.dumps(m.to_dict())))
    assert m2.same_layout(m) and m2.version == 3
    for (n, t), (n2, t2) in zip(named, unpack(arena, m2)):
        assert n == n2 and t2.dtype == t.dtype and torch.equal(t2, t)


def _sub(reg, name, **kw):
    return WeightSubscriber(reg, LocalTransport(name), name, chunk_bytes=kw.pop("chunk", 4096), heartbeat_s=0, **kw)


def test_publish_pull_tree_fanout():
    reg = WeightRegistry(fanout=1)
    pub = WeightPublisher(reg, LocalTransport("trainer"))
    v = pub.publish(weights_for(1))
    s1, s2, s3 = _sub(reg, "e1"), _sub(reg, "e2"), _sub(reg, "e3")
    for s in (s1, s2, s3):
        got = {}
        s.sync(lambda named: got.update({n: t.clone() for n, t in named}), v)
        assert torch.equal(got["w"], weights_for(1)[0][1]) and s.version == v
    # e1 read from the publisher; later readers preferred engines with spare fan-out
    assert s1.stats["sources"] == [PUBLISHER]
    assert s2.stats["sources"] == ["e1"]
    assert reg.status()["members"] == {"e1": 1, "e2": 1, "e3": 1}
    assert reg.wait_all(1, timeout=0.1)


def test_source_dies_mid_pull_survivor_completes():
    reg = WeightRegistry(fanout=4)
    pub = WeightPublisher(reg, LocalTransport("trainer"))
    pub.publish(weights_for(1, n=1 << 14))
    s1 = _sub(reg, "e1")
    s1.sync(lambda named: None)
    # e2 is assigned e1 (spare fan-out beats the publisher); e1 dies during the read
    t1 = s1.t
    orig = LocalTransport.read_batch
    calls = {"n": 0}

    def flaky(self, url, ops, dst, timeout_ms=None):
        calls["n"] += 1
        if url == t1.url and calls["n"] == 3:
            t1.kill()
        return orig(self, url, ops, dst, timeout_ms)
    LocalTransport.read_batch = flaky
    try:
        s2 = _sub(reg, "e2", window=1)
        got = {}
        s2.sync(lambda named: got.update({n: t.clone() for n, t in named}))
    finally:
        LocalTransport.read_batch = orig
    assert s2.stats["source_failures"] == 1 and s2.stats["sources"] == ["e1", PUBLISHER]
    assert torch.equal(got["w"], weights_for(1, n=1 << 14)[0][1])
    assert "e1" not in reg.status()["holders"]["1"]


def test_rolling_read_resumes_after_completed_prefix():
    reg = WeightRegistry()
    pub = WeightPublisher(reg, LocalTransport("trainer"))
    pub.publish(weights_for(2, n=8192))
    sub = _sub(reg, "e1", chunk=1024, window=2)
    seen = []
    orig = LocalTransport.read_batch
    state = {"fail": True}

    def once(self, url, ops, dst, timeout_ms=None):
        seen.extend(o[1] for o in ops)
        if state["fail"] and len(seen) >= 6:
            state["fail"] = False
            raise TransferError("injected")
        return orig(self, url, ops, dst, timeout_ms)
    LocalTransport.read_batch = once
    try:
        sub.pull()
    finally:
        LocalTransport.read_batch = orig
    # the failed window (offsets 4096, 5120) is read again, nothing before it
    assert seen[:6] == [0, 1024, 2048, 3072, 4096, 5120] and seen[6:8] == [4096, 5120]
    assert torch.equal(dict(sub.tensors())["w"], weights_for(2, n=8192)[0][1])


def test_join_catches_up_to_latest_and_double_buffer():
    reg = WeightRegistry()
    pub = WeightPublisher(reg, LocalTransport("trainer"), buffers=2, idle_timeout=0.2)
    for v in (1, 2, 3):
        pub.publish(weights_for(v))
    assert [a[1] for a in pub.arenas] == [3, 2]    # slot of v1 reused for v3
    late = _sub(reg, "late")
    assert late.sync(lambda n: None)["version"] == 3
    # a reader still assigned to v2 when the publisher reuses its slot is told its copy is stale
    src = reg.assign(version=3, member="slow")
    assert src["member"] in ("late", PUBLISHER)
    reg.assign(version=2, member="slow2")
    pub.publish(weights_for(4))                    # waits 0.2 s for v2's reader, then overwrites
    assert reg.release(version=2, source=PUBLISHER, member="slow2").get("stale") is True


def test_registry_over_http_and_expiry():
    srv = RegistryServer(WeightRegistry(member_ttl_s=0.3), host="127.0.0.1", expire_interval=0.05)
    try:
        cli = RegistryClient(f"http://127.0.0.1:{srv.port}")
        assert cli.join(member="m1", url="local://m1") == {"latest": None}
        pub = WeightPublisher(cli, LocalTransport("trainer-http"))
        pub.publish(weights_for(1))
        assert cli.get_latest()["version"] == 1
        with pytest.raises(RuntimeError, match="ValueError"):
            cli.publish(version=1, manifest={}, url="x", addr=0)
        with pytest.raises(AttributeError):
            cli.not_a_method
        assert cli.heartbeat(member="m1")["ok"]
        time.sleep(0.6)
        assert "m1" not in cli.status()["members"]
        assert cli.heartbeat(member="m1")["ok"] is False
    finally:
        srv.close()


def test_non_relay_member_frees_arena():
    reg = WeightRegistry()
    WeightPublisher(reg, LocalTransport("trainer")).publish(weights_for(1))
    s = _sub(reg, "nr", relay=False)
    s.sync(lambda n: None)
    assert s.arena is None and "nr" not in reg.status()["holders"]["1"]
    assert reg.status()["members"]["nr"] == 1


def test_host_arena_option(monkeypatch):
    reg = WeightRegistry()
    WeightPublisher(reg, LocalTransport("trainer")).publish(weights_for(1))
    monkeypatch.setenv("CONNEX_RL_ARENA", "host")
    s = _sub(reg, "h")
    s.pull()
    assert s.arena.device.type == "cpu"
    with pytest.raises(ValueError):
        _sub(reg, "bad", arena="gpu")


# ----------------------------------------------------------- rollout pool
def _run(coro):
    return asyncio.run(coro)


def test_pool_update_never_mixes_versions():
    async def main():
        pool = RolloutPool(version=1)
        insts = [FakeInstance(f"i{k}", tpot_s=0.0005) for k in range(3)]
        for i in insts:
            await pool.add(i)
        reqs = [{"seed": s, "max_tokens": 20} for s in range(30)]
        tasks = [asyncio.create_task(pool.generate(r)) for r in reqs]
        await asyncio.sleep(0.003)
        await pool.update(2, rolling=1)
        outs = await asyncio.gather(*tasks)
        for r, o in zip(reqs, outs):
            assert o["tokens"] == expected(r, float(o["version"]))
        assert pool.stats["completed"] == 30 and all(i.version == 2 for i in insts)
    _run(main())


def test_pool_abort_on_update_restarts_at_new_version():
    async def main():
        pool = RolloutPool(version=1, drain_timeout=0.005)
        inst = FakeInstance("i0", tpot_s=0.002)
        await pool.add(inst)
        r = {"seed": 5, "max_tokens": 50}
        t = asyncio.create_task(pool.generate(r))
        await asyncio.sleep(0.01)
        await pool.update(2)
        o = await t
        assert o["version"] == 2 and o["tokens"] == expected(r, 2.0)
        assert pool.stats["aborted_for_update"] == 1
    _run(main())


def test_pool_churn_death_resumes_on_same_version():
    async def main():
        pool = RolloutPool(version=1)
        a, b = FakeInstance("a", tpot_s=0.001), FakeInstance("b", tpot_s=0.001)
        await pool.add(a)
        r = {"seed": 9, "max_tokens": 40}
        t = asyncio.create_task(pool.generate(r))
        await asyncio.sleep(0.01)
        await pool.add(b)
        a.kill()
        o = await t
        assert o["instance"] == "b" and o["tokens"] == expected(r, 1.0)
        assert pool.stats["resumed"] == 1 and pool.stats["instance_failures"] == 1
        assert "a" not in pool.slots
    _run(main())


def test_fake_instance_updates_through_subscriber():
    reg = WeightRegistry()
    pub = WeightPublisher(reg, LocalTransport("trainer"))

    async def main():
        pub.publish(weights_for(1))
        pool = RolloutPool(version=1)
        inst = FakeInstance("s0", subscriber=_sub(reg, "s0"))
        await pool.add(inst)
        assert inst.w == 1.0
        pub.publish(weights_for(2))
        assert await pool.update(2) == 1
        o = await pool.generate({"seed": 1, "max_tokens": 5})
        assert o["tokens"] == expected({"seed": 1, "max_tokens": 5}, 2.0)
    _run(main())


# ------------------------------------------------------------- engine glue
def test_sglang_control_payload_and_loader(monkeypatch):
    import pickle
    from connex.rl import sglang_ext
    srv = RegistryServer(WeightRegistry(), host="127.0.0.1")
    try:
        url = f"http://127.0.0.1:{srv.port}"
        WeightPublisher(RegistryClient(url), LocalTransport("trainer-sg")).publish(weights_for(4), version=4)
        payload = sglang_ext.control_payload(url, 4, "sg", transport="local")
        ctl = sglang_ext.parse_control(pickle.loads(pickle.dumps(payload)))
        assert ctl["version"] == 4 and ctl["transport"] == "local"

        class Model:
            got = None

            def load_weights(self, named):
                self.got = dict(named)
        monkeypatch.setenv("CONNEX_RL_DEVICE", "cpu")
        sglang_ext.reset_subscriber()
        m = Model()
        sglang_ext.connex_load(m, payload)
        assert torch.equal(m.got["b"], weights_for(4)[1][1]) and sglang_ext.last_stats["version"] == 4
        m2 = Model()
        sglang_ext.connex_load(m2, [("x", torch.ones(2))])   # plain tensors pass through
        assert torch.equal(m2.got["x"], torch.ones(2))
        sglang_ext.reset_subscriber()
    finally:
        srv.close()


class _FakeHTTP:
    """Minimal threaded HTTP server recording POSTs and answering per path."""

    def __init__(self, answers):
        from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
        calls = self.calls = []

        class H(BaseHTTPRequestHandler):
            def log_message(self, *a):
                pass

            def do_POST(self):
                n = int(self.headers.get("Content-Length") or 0)
                body = json.loads(self.rfile.read(n) or b"null")
                calls.append((self.path.split("?")[0], body))
                code, out = answers.get(self.path.split("?")[0], (200, {}))
                data = json.dumps(out).encode()
                self.send_response(code)
                self.send_header("Content-Length", str(len(data)))
                self.end_headers()
                self.wfile.write(data)
        self.srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
        threading.Thread(target=self.srv.serve_forever, daemon=True).start()
        self.url = f"http://127.0.0.1:{self.srv.server_address[1]}"

    def close(self):
        self.srv.shutdown()
        self.srv.server_close()


def test_vllm_and_sglang_instance_protocols():
    from connex.rl.engines import SGLangInstance, VLLMInstance
    from connex.rl.rollout import Aborted, InstanceDead
    fv = _FakeHTTP({"/v1/completions": (200, {"choices": [{"token_ids": [1, 2, 3], "finish_reason": "length"}]})})
    fs = _FakeHTTP({"/generate": (200, {"output_ids": [4, 5], "meta_info": {"finish_reason": {"type": "abort"}}}),
                    "/begin_weight_update": (404, {})})

    async def main():
        v = VLLMInstance("v", fv.url, "m", "http://reg")
        assert (await v.generate({"prompt_ids": [9], "max_tokens": 3}))["tokens"] == [1, 2, 3]
        await v.update(7)
        assert v.version == 7
        assert [c[0] for c in fv.calls[1:]] == ["/init_weight_transfer_engine", "/start_weight_update",
                                                "/update_weights", "/finish_weight_update"]
        await v.close()
        s = SGLangInstance("s", fs.url, "m", "http://reg", tp_size=2)
        with pytest.raises(Aborted):
            await s.generate({"prompt_ids": [1], "max_tokens": 2, "seed": 3})
        await s.update(3)
        upd = [c for c in fs.calls if c[0] == "/update_weights_from_tensor"][0][1]
        assert len(upd["serialized_named_tensors"]) == 2 and upd["weight_version"] == "3"
        await s.close()
        dead = VLLMInstance("d", "http://127.0.0.1:9", "m", "http://reg", timeout=2)
        with pytest.raises(InstanceDead):
            await dead.generate({"prompt_ids": [1], "max_tokens": 1})
        await dead.close()
    try:
        _run(main())
    finally:
        fv.close()
        fs.close()

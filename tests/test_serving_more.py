"""More serving behaviours on CPU against the deterministic fake backends:
passthrough without failures, usage only when asked, refused connects,
several failures in one stream, non-streaming resume, batch prompts that
cannot be resumed, logprobs=0, the prefill of a long prompt that is not cut
by the idle timer, new PD members kept out until probed, a decode death
after the prefill instance is gone (re-prefill of the extended prompt), and
session fields that never reach the backend."""
import asyncio

import aiohttp

from connex.agents import SessionProxy
from connex.serving.fake_backend import FakeBackend, FakePDBackend, reference
from connex.serving.pd_router import ElasticPool, PDRouter
from connex.serving.proxy import Pool
from tests.helpers import free_port
from tests.test_serving import _proxy, _run, _serve, _stream, _text


def test_steady_state_passthrough_and_usage_only_when_asked():
    async def main():
        a = FakeBackend()
        ua = await a.start()
        pr, url = await _serve(_proxy([ua]).app())
        try:
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t3 t4", "max_tokens": 6})
            assert done and _text(chunks) == reference("t3 t4", 6)[1]
            assert all(not c.get("usage") for c in chunks)            # not requested: none
            assert len(a.requests) == 1 and a.requests[0]["max_tokens"] == 6
            chunks, _ = await _stream(url, "/v1/completions", {"prompt": "t3 t4", "max_tokens": 6,
                                                               "stream_options": {"include_usage": True}})
            assert chunks[-1]["usage"]["completion_tokens"] == 6
        finally:
            await pr.cleanup()
            await a.stop()
    _run(main())


def test_refused_connect_is_retried_elsewhere():
    async def main():
        a = FakeBackend()
        ua = await a.start()
        dead = f"http://127.0.0.1:{free_port()}"                    # nothing listens there
        p = _proxy([dead, ua])
        pr, url = await _serve(p.app())
        try:
            for _ in range(3):
                chunks, done = await _stream(url, "/v1/completions", {"prompt": [1, 5], "max_tokens": 4})
                assert done and _text(chunks) == reference([1, 5], 4)[1]
            assert len(a.requests) == 3
        finally:
            await pr.cleanup()
            await a.stop()
    _run(main())


def test_two_failures_at_different_points_in_one_stream():
    async def main():
        a, b = FakeBackend(), FakeBackend()
        ua, ub = await a.start(), await b.start()
        a.fail, a.fail_count = ("reset", 3), 1
        b.fail, b.fail_count = ("reset", 2), 1
        p = _proxy([ua, ub])
        pr, url = await _serve(p.app())
        try:
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t1 t9", "max_tokens": 14})
            assert done and _text(chunks) == reference("t1 t9", 14)[1]
            assert p.stats["resumes"] >= 2 and len({c["id"] for c in chunks}) == 1
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_non_streaming_request_is_resumed_and_aggregated():
    async def main():
        a, b = FakeBackend(), FakeBackend()
        ua, ub = await a.start(), await b.start()
        for x in (a, b):
            x.fail, x.fail_count = ("reset", 4), 1
        pr, url = await _serve(_proxy([ua, ub]).app())
        try:
            async with aiohttp.ClientSession() as s:
                async with s.post(url + "/v1/completions", json={"prompt": "t8", "max_tokens": 9}) as r:
                    out = await r.json()
            assert r.status == 200 and out["choices"][0]["text"] == reference("t8", 9)[1]
            assert out["usage"]["completion_tokens"] == 9
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_batch_prompt_is_passed_through_not_resumed():
    async def main():
        a = FakeBackend()
        ua = await a.start()
        p = _proxy([ua])
        pr, url = await _serve(p.app())
        try:
            async with aiohttp.ClientSession() as s:
                async with s.post(url + "/v1/completions", json={"prompt": ["t1", "t2"], "max_tokens": 3}) as r:
                    await r.read()
            req = a.requests[-1]
            assert req["prompt"] == ["t1", "t2"]
            assert "return_token_ids" not in req and "return_tokens_as_token_ids" not in req
        finally:
            await pr.cleanup()
            await a.stop()
    _run(main())


def test_logprobs_zero_reaches_the_client():
    async def main():
        a = FakeBackend()
        ua = await a.start()
        pr, url = await _serve(_proxy([ua]).app())
        try:
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t2", "max_tokens": 3, "logprobs": 0})
            assert done and a.requests[-1]["logprobs"] == 0
            lps = [ch.get("logprobs") for c in chunks for ch in c.get("choices") or []]
            assert any(lp for lp in lps)
        finally:
            await pr.cleanup()
            await a.stop()
    _run(main())


def test_slow_first_token_is_not_cut_by_the_idle_timer():
    async def main():
        a = FakeBackend(ttft_ms=600)                                 # a long prefill
        ua = await a.start()
        p = _proxy([ua], idle_timeout=0.2)
        pr, url = await _serve(p.app())
        try:
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t6", "max_tokens": 3})
            assert done and _text(chunks) == reference("t6", 3)[1] and len(a.requests) == 1
        finally:
            await pr.cleanup()
            await a.stop()
    _run(main())


def test_new_pd_member_takes_no_traffic_until_probed():
    async def main():
        kv = {}
        p0, d0 = FakePDBackend("prefill", kv), FakePDBackend("decode", kv)
        up, ud = await p0.start(), await d0.start()
        dpool = ElasticPool([], probe_new=True)
        dpool.set_urls([ud])
        assert dpool.healthy_urls() == []                          # listed, not probed yet
        router = PDRouter(ElasticPool([up], probe_new=False), dpool, probe_interval=0.05, idle_timeout=0.5)
        pr, url = await _serve(router.app())
        try:
            for _ in range(100):
                if dpool.healthy_urls():
                    break
                await asyncio.sleep(0.02)
            assert dpool.healthy_urls() == [ud]                    # one good probe admits it
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t3", "max_tokens": 3})
            assert done and _text(chunks) == reference("t3", 3)[1]
        finally:
            await pr.cleanup()
            await p0.stop()
            await d0.stop()
    _run(main())


def test_decode_death_after_prefill_is_gone_reprefills_the_extended_prompt():
    async def main():
        kv = {}
        p0 = FakePDBackend("prefill", kv)
        d0, d1 = FakePDBackend("decode", kv), FakePDBackend("decode", kv)
        up, u0, u1 = await p0.start(), await d0.start(), await d1.start()
        for d in (d0, d1):
            d.fail, d.fail_count = ("reset", 3), 1
        router = PDRouter(ElasticPool([up], probe_new=False), ElasticPool([u0, u1], probe_new=False),
                          probe_interval=0, idle_timeout=0.5)
        pr, url = await _serve(router.app())
        try:
            real = d0._generate, d1._generate
            state = {"cleared": False}

            def drop_kv_once(gen):
                async def f(req, b, ids, chat):
                    if router.stats.get("kv_repulls", 0) >= 1 and not state["cleared"]:
                        state["cleared"] = True
                        kv.clear()                                   # the prefill's hold is gone too
                    return await gen(req, b, ids, chat)
                return f
            d0._generate = drop_kv_once(real[0])
            d1._generate = drop_kv_once(real[1])
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t4 t5", "max_tokens": 10})
            assert done and _text(chunks) == reference("t4 t5", 10)[1]
            assert router.stats["kv_reprefills"] >= 1
            # the re-prefill carried the prompt plus the tokens already streamed
            lens = [len(r["prompt"]) for r in p0.requests if isinstance(r.get("prompt"), list)]
            assert lens and max(lens) > 3
        finally:
            await pr.cleanup()
            for x in (p0, d0, d1):
                await x.stop()
    _run(main())


def test_session_fields_do_not_reach_the_backend():
    async def main():
        a = FakeBackend()
        ua = await a.start()
        sp = SessionProxy(Pool([ua]), probe_interval=0, idle_timeout=0.5)
        pr, url = await _serve(sp.app())
        try:
            msgs = [{"role": "user", "content": "t1"}]
            await _stream(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 2, "session_id": "z"})
            await _stream(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 2},
                          headers={"X-Connex-Session": "z"})
            assert all("session_id" not in r for r in a.requests) and sp.sessions["z"].url == ua
        finally:
            await pr.cleanup()
            await a.stop()
    _run(main())

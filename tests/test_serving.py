"""Serving layer on CPU: resume proxy (retry, token-id and chat resume, idle
stall, passthrough, aggregate), PD router (prefill retry, KV re-pull after a
decode death, re-prefill after a failed hand-off, drain, failure events,
SGLang pairing) and agent sessions (sticky routing, migration, failover),
all against the deterministic fake backends."""
import asyncio
import json
import os
import tempfile

import aiohttp
import pytest
from aiohttp import web

from connex.agents import SessionProxy
from connex.serving.fake_backend import (FakeBackend, FakePDBackend, FakeSGLangPDBackend, chat_ids, detok,
                                         next_token, reference)
from connex.serving.pd_router import ElasticPool, PDRouter
from connex.serving.proxy import Pool, Proxy


async def _serve(app):
    runner = web.AppRunner(app, shutdown_timeout=0.1)
    await runner.setup()
    site = web.TCPSite(runner, "127.0.0.1", 0)
    await site.start()
    return runner, f"http://127.0.0.1:{site._server.sockets[0].getsockname()[1]}"


async def _stream(url, path, body, headers=None):
    """(chunks, saw_done) of a streamed request."""
    chunks, done = [], False
    async with aiohttp.ClientSession() as s:
        async with s.post(url + path, json={**body, "stream": True}, headers=headers or {}) as r:
            assert r.status == 200, await r.text()
            async for line in r.content:
                line = line.strip()
                if not line.startswith(b"data:"):
                    continue
                d = line[5:].strip()
                if d == b"[DONE]":
                    done = True
                    break
                chunks.append(json.loads(d))
    return chunks, done


def _text(chunks, chat=False):
    out = []
    for c in chunks:
        for ch in c.get("choices") or []:
            out.append((ch.get("delta") or {}).get("content") or "" if chat else ch.get("text") or "")
    return "".join(out)


def _run(coro):
    return asyncio.run(asyncio.wait_for(coro, 60))


def _proxy(urls, **kw):
    kw.setdefault("probe_interval", 0)
    kw.setdefault("idle_timeout", 0.5)
    return Proxy(Pool(urls, blacklist_s=kw.pop("blacklist_s", 5.0)), **kw)


def test_proxy_resumes_after_reset_with_token_ids():
    async def main():
        a, b = FakeBackend(), FakeBackend()
        ua, ub = await a.start(), await b.start()
        for x in (a, b):            # each replica breaks once, after 5 tokens of its stream
            x.fail, x.fail_count = ("reset", 5), 1
        pr, url = await _serve(_proxy([ua, ub]).app())
        try:
            body = {"model": "fake", "prompt": "t5 t6 t7", "max_tokens": 12,
                    "stream_options": {"include_usage": True}}
            chunks, done = await _stream(url, "/v1/completions", body)
            assert done
            ids, text = reference("t5 t6 t7", 12)
            assert _text(chunks) == text
            assert len({c["id"] for c in chunks}) == 1
            assert chunks[-1]["usage"]["completion_tokens"] == 12
            assert chunks[-1]["usage"]["prompt_tokens"] == 4
            reqs = sorted(a.requests + b.requests, key=lambda r: -r["max_tokens"])
            assert [r["max_tokens"] for r in reqs] == [12, 7, 2]
            assert reqs[1]["prompt"][-5:] == ids[:5] and reqs[2]["prompt"][-10:] == ids[:10]
            assert all("token_ids" not in (c["choices"] or [{}])[0] for c in chunks)
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_proxy_retries_before_first_token_and_idle_stall_resume():
    async def main():
        a, b = FakeBackend(), FakeBackend()
        ua, ub = await a.start(), await b.start()
        pr, url = await _serve(_proxy([ua, ub], idle_timeout=0.3).app())
        try:
            a.fail, a.fail_count = ("http500", 0), 1
            b.fail, b.fail_count = ("stall", 3), 1
            body = {"model": "fake", "prompt": [1, 9, 9], "max_tokens": 8}
            chunks, done = await _stream(url, "/v1/completions", body)
            assert done and _text(chunks) == reference([1, 9, 9], 8)[1]
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_proxy_chat_resume_aggregate_and_passthrough():
    async def main():
        a, b = FakeBackend(), FakeBackend()
        ua, ub = await a.start(), await b.start()
        for x in (a, b):
            x.fail, x.fail_count = ("reset", 3), 1
        p = _proxy([ua, ub])
        pr, url = await _serve(p.app())
        try:
            msgs = [{"role": "user", "content": "t3 t4"}]
            async with aiohttp.ClientSession() as s:
                async with s.post(url + "/v1/chat/completions",
                                  json={"model": "fake", "messages": msgs, "max_tokens": 6}) as r:
                    out = await r.json()
                assert r.status == 200
                content = out["choices"][0]["message"]["content"]
                assert out["usage"]["completion_tokens"] == 6 and content.count(" t") == 6
                # continuation went through continue_final_message with the partial reply
                cont = [r for r in a.requests + b.requests if r.get("continue_final_message")]
                assert len(cont) == 1 and cont[0]["messages"][-1]["role"] == "assistant"
                async with s.post(url + "/v1/completions", json={"model": "fake", "prompt": "x", "max_tokens": 0}) \
                        as r:
                    assert r.status == 400          # client error passes through, no retry
            assert p.stats["resumes"] == 1
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_proxy_all_down_502_and_file_removal():
    async def main():
        a = FakeBackend()
        ua = await a.start()
        with tempfile.TemporaryDirectory() as d:
            f = os.path.join(d, "eps")
            with open(f, "w") as fh:
                fh.write("http://127.0.0.1:9\n" + ua + "\n")
            pool = Pool([], f, blacklist_s=5)
            p = Proxy(pool, probe_interval=0, idle_timeout=0.5, max_attempts=2)
            pool.reload()
            assert pool.order == ["http://127.0.0.1:9", ua]
            with open(f, "w") as fh:
                fh.write(ua + "\n")
            pool.reload()
            assert pool.order == [ua]
            pr, url = await _serve(p.app())
            try:
                await a.stop()
                async with aiohttp.ClientSession() as s:
                    async with s.post(url + "/v1/completions", json={"prompt": "t1", "max_tokens": 2}) as r:
                        assert r.status == 502
                    async with s.get(url + "/health") as r:
                        assert r.status == 503
            finally:
                await pr.cleanup()
    _run(main())


def _pd(prefills, decodes, **kw):
    kw.setdefault("probe_interval", 0)
    kw.setdefault("idle_timeout", 0.5)
    return PDRouter(ElasticPool(prefills, probe_new=False), ElasticPool(decodes, probe_new=False), **kw)


def test_pd_router_flow_retry_and_repull():
    async def main():
        kv = {}
        p0, p1 = FakePDBackend("prefill", kv), FakePDBackend("prefill", kv)
        d0, d1 = FakePDBackend("decode", kv), FakePDBackend("decode", kv)
        urls = [await x.start() for x in (p0, p1, d0, d1)]
        for x in (p0, p1):      # whichever prefill goes first fails once
            x.fail, x.fail_count = ("http500", 0), 1
        for x in (d0, d1):      # each decode dies once, 4 tokens into its stream
            x.fail, x.fail_count = ("reset", 4), 1
        router = _pd(urls[:2], urls[2:])
        pr, url = await _serve(router.app())
        try:
            body = {"model": "fake", "prompt": "t10 t11", "max_tokens": 10}
            chunks, done = await _stream(url, "/v1/completions", body)
            assert done and _text(chunks) == reference("t10 t11", 10)[1]
            assert router.stats["prefill_retries"] >= 1 and router.stats["prefills"] == 1
            # both decode deaths resumed elsewhere by re-pulling the held prompt KV (no re-prefill)
            assert router.stats["kv_repulls"] == 2 and d0.pulls + d1.pulls == 3
            assert router.stats["kv_reprefills"] == 0
        finally:
            await pr.cleanup()
            for x in (p0, p1, d0, d1):
                await x.stop()
    _run(main())


def test_pd_router_reprefill_when_handoff_fails_and_drain():
    async def main():
        kv = {}
        p0, p1 = FakePDBackend("prefill", kv), FakePDBackend("prefill", kv)
        d0 = FakePDBackend("decode", kv)
        urls = [await x.start() for x in (p0, p1, d0)]
        router = _pd(urls[:2], urls[2:])
        pr, url = await _serve(router.app())
        try:
            real = d0._generate
            calls = {"n": 0}

            async def lose_first(req, b, ids, chat):
                calls["n"] += 1
                if calls["n"] == 1:     # the hold vanished: KV load fails, decode itself alive
                    kv.clear()
                return await real(req, b, ids, chat)
            d0._generate = lose_first
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t2", "max_tokens": 5})
            assert done and _text(chunks) == reference("t2", 5)[1]
            assert router.stats["kv_reprefills"] == 1 and router.stats["prefills"] == 2
            async with aiohttp.ClientSession() as s:
                async with s.post(url + "/pd/drain", json={"url": urls[0], "role": "prefill"}) as r:
                    assert r.status == 200
                async with s.get(url + "/pd/pools") as r:
                    pools = await r.json()
            assert [x["url"] for x in pools["prefill"] if not x.get("drained")] == [urls[1]]
            # a failure event for a known member cuts it at once
            router._members[("decode", 0)] = urls[2]
            from connex.pd.membership import PD_STAGE
            ev = {"payload": {"reason": "lease_expired", "lid": {"stage_idx": PD_STAGE["decode"], "replica_idx": 0}}}
            assert router.on_failure_event(ev) is True
            assert router.on_failure_event({"payload": {"reason": "group_left"}}) is False
        finally:
            await pr.cleanup()
            for x in (p0, p1, d0):
                await x.stop()
    _run(main())


def test_pd_router_sglang_pairing():
    async def main():
        rooms = {}
        p0, d0 = FakeSGLangPDBackend("prefill", rooms), FakeSGLangPDBackend("decode", rooms)
        up, ud = await p0.start(), await d0.start()
        router = _pd([up], [ud], engine="sglang")
        pr, url = await _serve(router.app())
        try:
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t7", "max_tokens": 4})
            assert done and _text(chunks) == reference("t7", 4)[1] and p0.prefills == 1
            assert "bootstrap_room" in d0.requests[-1]
        finally:
            await pr.cleanup()
            await p0.stop()
            await d0.stop()
    _run(main())


def test_session_sticky_migrate_and_failover():
    async def main():
        a, b = FakeBackend(tpot_ms=2), FakeBackend(tpot_ms=2)
        ua, ub = await a.start(), await b.start()
        sp = SessionProxy(Pool([ua, ub]), probe_interval=0, idle_timeout=0.5)
        pr, url = await _serve(sp.app())
        try:
            msgs = [{"role": "user", "content": "t1 t2"}]
            for _ in range(2):
                await _stream(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 3, "session_id": "s1"})
            first = sp.sessions["s1"].url
            assert len([r for r in (a.requests + b.requests)]) == 2
            assert (a if first == ua else b).requests and not (b if first == ua else a).requests
            other = ub if first == ua else ua
            rec = await sp.migrate("s1", other)
            assert rec["epoch"] == 1 and rec["mode"] == "reprefill" and sp.sessions["s1"].url == other
            prefilled = (b if other == ub else a).requests[-1]
            assert prefilled["max_tokens"] == 1 and prefilled["messages"][-1]["role"] == "assistant"
            # placement dies: the next turn fails over
            await (b if other == ub else a).stop()
            chunks, done = await _stream(url, "/v1/chat/completions",
                                         {"messages": msgs, "max_tokens": 3}, headers={"X-Connex-Session": "s1"})
            assert done and sp.stats["failovers"] == 1 and sp.sessions["s1"].url == first
        finally:
            await pr.cleanup()
            await a.stop()
            await b.stop()
    _run(main())


def test_fake_model_is_prefix_consistent():
    ids = chat_ids([{"role": "user", "content": "t1"}])
    assert ids[0] == 1 and ids[-2:] == [2, 3]
    full, _ = reference([1, 2, 3], 6)
    part, _ = reference([1, 2, 3] + full[:2], 4)
    assert full[2:] == part and detok(next_token([5])).startswith(" t")

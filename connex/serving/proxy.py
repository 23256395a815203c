"""Resume proxy: an OpenAI-API front that hides replica deaths from clients
(reference ``connex/serving/proxy.py:84-764``).

* **Replicas** come from ``--endpoints`` and/or an endpoints file (re-read
  every ``--reload-interval`` s; an URL removed from the file counts as
  dead).  A prober GETs ``/v1/models`` on fresh connections; two failed
  probes, a connect error or a broken stream blacklist a replica for
  ``--blacklist-s``.  The least-loaded healthy replica is picked.
* **Before the first token** a failed attempt (refused, reset, 5xx, the
  replica declared dead while we wait) is retried elsewhere.  No idle timer
  runs before the first token, so a long prefill is never cut; the wait ends
  only when the replica is declared dead (or an optional first-token cap).
* **After k tokens** (reset, EOF without ``[DONE]``, no chunk for
  ``--idle-timeout`` s) the request resumes on another replica: completions
  from token ids (``prompt_ids + generated_ids``; the proxy asks for
  ``return_token_ids`` / id logprobs and strips them again), chat through
  ``continue_final_message``; ``max_tokens``/``min_tokens`` shrink by k.  The
  client sees one stream with one ``id`` and a usage block counting the
  original prompt and all completion tokens.

Every backend call streams; non-streaming clients get the aggregate.
:meth:`Proxy.move` cuts a request over on purpose (planned migration).

    python -m connex.serving.proxy --port 5199 --endpoints http://a:5100,http://b:5101
"""
from __future__ import annotations

import argparse
import asyncio
import json
import logging
import time
from typing import Dict, List, Optional

import aiohttp
from aiohttp import web

log = logging.getLogger("connex.proxy")

RETRYABLE = (aiohttp.ClientError, asyncio.TimeoutError, ConnectionError, OSError)


def _loads(b):
    return json.loads(b)


def _sse(obj) -> bytes:
    return b"data: " + json.dumps(obj, separators=(",", ":")).encode() + b"\n\n"


class StreamBroken(Exception):
    pass


class HTTPPassthrough(Exception):
    """A client error from the backend (4xx before any token): forwarded as is."""

    def __init__(self, status, payload, ctype):
        super().__init__(f"HTTP {status}")
        self.status, self.payload, self.ctype = status, payload, ctype or "application/json"


class UpstreamFailed(Exception):
    def __init__(self, msg, st):
        super().__init__(msg)
        self.st = st


# ------------------------------------------------------------------ pool
class Endpoint:
    __slots__ = ("url", "bad_until", "inflight", "dead")

    def __init__(self, url: str):
        self.url = url.rstrip("/")
        self.bad_until = 0.0
        self.inflight = 0
        self.dead = asyncio.Event()     # set while blacklisted: wakes its waiters

    def healthy(self, now: float) -> bool:
        return now >= self.bad_until


class Pool:
    def __init__(self, urls=(), endpoints_file: Optional[str] = None, blacklist_s: float = 5.0):
        self.eps: Dict[str, Endpoint] = {}
        self.order: List[str] = []
        self.file = endpoints_file
        self.blacklist_s = blacklist_s
        self._rr = 0
        self.set_urls(urls)

    def set_urls(self, urls) -> None:
        urls = [u.strip().rstrip("/") for u in urls if u.strip()]
        for u in urls:
            self.eps.setdefault(u, Endpoint(u))
        self.order = urls

    def _file_urls(self) -> Optional[List[str]]:
        try:
            with open(self.file) as f:
                return [x.strip().rstrip("/") for x in f if x.strip()]
        except OSError:
            return None

    def reload(self) -> None:
        if not self.file:
            return
        urls = self._file_urls()
        if not urls:
            return
        gone = [u for u in self.order if u not in urls]
        self.set_urls(urls)
        for u in gone:      # removed (e.g. by a supervisor that saw it die): dead now
            self.mark_bad(self.eps[u], "removed from endpoints file")

    def mark_bad(self, ep: Endpoint, why: str = "") -> None:
        if ep.healthy(time.monotonic()):
            log.warning("blacklisting %s for %.1fs: %s", ep.url, self.blacklist_s, why)
        ep.bad_until = time.monotonic() + self.blacklist_s
        ep.dead.set()

    def mark_good(self, ep: Endpoint) -> None:
        if ep.bad_until:
            ep.bad_until = 0.0
            ep.dead = asyncio.Event()

    def pick(self, exclude=()) -> Optional[Endpoint]:
        now = time.monotonic()
        cands = [self.eps[u] for u in self.order if u not in exclude]
        if not cands:
            return None
        ok = [e for e in cands if e.healthy(now)]
        if not ok:          # last resort: the one whose blacklist ends first
            return min(cands, key=lambda e: e.bad_until)
        for e in ok:
            if e.bad_until:     # blacklist lapsed without a probe: re-arm
                self.mark_good(e)
        self._rr += 1
        rot = ok[self._rr % len(ok):] + ok[:self._rr % len(ok)]
        return min(rot, key=lambda e: e.inflight)


def _ids_from_logprobs(lp, chat: bool):
    if not lp:
        return None
    toks = [c.get("token") for c in lp.get("content") or []] if chat else lp.get("tokens")
    if not toks:
        return None
    out = []
    for t in toks:
        if not isinstance(t, str) or not t.startswith("token_id:"):
            return None
        out.append(int(t[len("token_id:"):]))
    return out


# --------------------------------------------------------------- resumer
class Resumer:
    """One client request across its backend attempts."""

    def __init__(self, proxy: "Proxy", kind: str, body: dict):
        self.p = proxy
        self.kind = kind
        self.chat = kind == "chat"
        self.body = body
        so = body.get("stream_options") or {}
        self.client_usage = bool(so.get("include_usage"))
        self.client_cont_usage = bool(so.get("continuous_usage_stats"))
        prompt = body.get("prompt")
        single = body.get("n") in (None, 1) and body.get("best_of") in (None, 1)
        text_or_ids = isinstance(prompt, str) or (isinstance(prompt, list) and bool(prompt)
                                                  and isinstance(prompt[0], int))
        self.resumable = single and (self.chat or text_or_ids)
        lp = body.get("logprobs")
        self.client_lp = lp is not None and lp is not False      # logprobs=0 asks for them too
        self.use_ids = (self.resumable and not self.chat and proxy.token_ids
                        and (not self.client_lp or bool(body.get("return_tokens_as_token_ids"))))
        self.inject_lp = self.use_ids and not self.client_lp
        self.ids: List[int] = []
        self.text: List[str] = []
        self.k = 0
        self.prompt_tokens = None
        self.prompt_ids = prompt if isinstance(prompt, list) else None
        self.rid = self.created = None
        self.model = body.get("model")
        self.finish = self.stop_reason = None
        self.attempts = 0
        self.sent_role = False
        self.resp = None
        self.ep = None
        self.moved = False

    async def build(self, ep: Endpoint) -> dict:
        b = dict(self.body)
        b["stream"] = True
        b["stream_options"] = {"include_usage": True, "continuous_usage_stats": True}
        if self.inject_lp:
            b["logprobs"] = True if self.chat else 0
            b["return_tokens_as_token_ids"] = True
        if self.use_ids:
            b["return_token_ids"] = True
        if self.k == 0:
            return b
        for key in ("max_tokens", "max_completion_tokens"):
            if b.get(key) is not None:
                b[key] -= self.k
        if b.get("min_tokens"):
            b["min_tokens"] = max(0, b["min_tokens"] - self.k)
        done_text = "".join(self.text)
        if self.chat:
            msgs = [dict(m) for m in b["messages"]]
            if b.get("continue_final_message") and msgs and msgs[-1].get("role") == "assistant":
                msgs[-1]["content"] = (msgs[-1].get("content") or "") + done_text
            else:
                msgs.append({"role": "assistant", "content": done_text})
            b.update(messages=msgs, add_generation_prompt=False, continue_final_message=True)
            return b
        b["echo"] = False
        if self.use_ids and len(self.ids) == self.k:
            if self.prompt_ids is None:
                self.prompt_ids = await self.p.tokenize(ep, self.model, self.body["prompt"])
            if self.prompt_ids is not None:
                b["prompt"] = list(self.prompt_ids) + self.ids
                return b
        if isinstance(b["prompt"], str):
            b["prompt"] += done_text
            return b
        raise StreamBroken("cannot resume a token-id prompt without the generated ids")

    def can_resume(self) -> bool:
        return self.k == 0 or self.resumable

    def remaining(self):
        m = self.body.get("max_tokens")
        if m is None:
            m = self.body.get("max_completion_tokens")
        return None if m is None else m - self.k

    def on_chunk(self, c: dict, base_k: int):
        """Account one backend chunk; returns the chunk for the client or None."""
        usage = c.get("usage")
        choices = c.get("choices") or []
        if usage and base_k == 0 and self.prompt_tokens is None:
            self.prompt_tokens = usage.get("prompt_tokens")
        if not choices:             # trailing usage-only chunk: ours replaces it
            if usage and usage.get("completion_tokens") is not None:
                self.k = max(self.k, base_k + usage["completion_tokens"])
            return None
        if self.rid is None:
            self.rid, self.created = c.get("id"), c.get("created")
            self.model = c.get("model", self.model)
        ch = choices[0]
        if len(choices) > 1 or ch.get("index", 0) != 0:
            self.resumable = False
        if self.chat:
            delta = ch.get("delta") or {}
            piece = delta.get("content") or ""
            if not piece and ch.get("finish_reason") is None and "role" in delta:
                if self.sent_role:
                    return None     # role preamble of a retried / resumed stream
                self.sent_role = True
        else:
            piece = ch.get("text") or ""
        ids = ch.get("token_ids") or (_ids_from_logprobs(ch.get("logprobs"), self.chat) if self.use_ids else None)
        if usage and usage.get("completion_tokens") is not None:
            self.k = base_k + usage["completion_tokens"]
        elif ids:
            self.k += len(ids)
        elif piece:
            self.k += 1
        if self.use_ids:
            if ids:
                self.ids.extend(ids)
            if len(self.ids) != self.k:
                self.use_ids = False    # lost count: resume from text instead
        self.text.append(piece)
        if ch.get("finish_reason") is not None:
            self.finish, self.stop_reason = ch["finish_reason"], ch.get("stop_reason")
        c["id"], c["created"], c["model"] = self.rid, self.created, self.model
        if self.inject_lp:
            ch["logprobs"] = None
        if "token_ids" in ch and not self.body.get("return_token_ids"):
            del ch["token_ids"]
        if self.client_cont_usage:
            c["usage"] = self.usage()
        elif "usage" in c:
            c["usage"] = None
        return c

    def usage(self) -> dict:
        pt = self.prompt_tokens
        if pt is None and self.prompt_ids is not None:
            pt = len(self.prompt_ids)
        return {"prompt_tokens": pt, "completion_tokens": self.k, "total_tokens": (pt or 0) + self.k}


# ----------------------------------------------------------------- proxy
class Proxy:
    resumer_cls = Resumer

    def __init__(self, pool: Pool, idle_timeout: float = 2.5, connect_timeout: float = 2.0, max_attempts: int = 4,
                 probe_interval: float = 1.0, token_ids: bool = True, first_token_timeout: Optional[float] = None):
        self.pool = pool
        self.idle_timeout = idle_timeout
        self.first_token_timeout = first_token_timeout
        self.connect_timeout = connect_timeout
        self.max_attempts = max_attempts
        self.probe_interval = probe_interval
        self.token_ids = token_ids
        self.reload_interval = 1.0
        self.session: Optional[aiohttp.ClientSession] = None
        self.probe_session: Optional[aiohttp.ClientSession] = None
        self.stats = {"requests": 0, "retries": 0, "resumes": 0, "failed": 0}
        self._bg: List[asyncio.Task] = []

    def app(self) -> web.Application:
        app = web.Application(client_max_size=64 << 20)
        app.router.add_post("/v1/completions", self.handle_completions)
        app.router.add_post("/v1/chat/completions", self.handle_chat)
        app.router.add_get("/v1/models", self.handle_models)
        app.router.add_get("/health", self.handle_health)
        app.router.add_get("/proxy/stats", self.handle_stats)
        app.on_startup.append(self._startup)
        app.on_cleanup.append(self._cleanup)
        return app

    async def _startup(self, app=None):
        self.session = aiohttp.ClientSession(
            connector=aiohttp.TCPConnector(limit=0, ttl_dns_cache=300),
            timeout=aiohttp.ClientTimeout(total=None, sock_connect=self.connect_timeout),
            auto_decompress=False, trust_env=False)
        self.probe_session = aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=0, force_close=True),
                                                   trust_env=False)
        if self.pool.file:
            self.pool.reload()
            self._bg.append(asyncio.create_task(self._every(self.reload_interval, self.pool.reload)))
        if self.probe_interval:
            self._bg.append(asyncio.create_task(self._probe_loop()))

    async def _cleanup(self, app=None):
        for t in self._bg:
            t.cancel()
        await self.session.close()
        await self.probe_session.close()

    async def _every(self, s: float, fn) -> None:
        while True:
            await asyncio.sleep(s)
            fn()

    async def _probe_loop(self):
        while True:
            await asyncio.sleep(self.probe_interval)
            eps = [e for e in list(self.pool.eps.values()) if e.url in self.pool.order]
            await asyncio.gather(*(self._probe(e) for e in eps), return_exceptions=True)

    async def _alive(self, ep: Endpoint, timeout: float = 2.0) -> bool:
        try:
            async with self.probe_session.get(ep.url + "/v1/models",
                                              timeout=aiohttp.ClientTimeout(total=timeout)) as r:
                return r.status == 200
        except RETRYABLE:
            return False

    async def _probe(self, ep: Endpoint) -> None:
        # two failures in a row: a busy but alive server keeps its prefills
        if await self._alive(ep) or await self._alive(ep):
            self.pool.mark_good(ep)
        else:
            self.pool.mark_bad(ep, "probe failed twice")

    async def tokenize(self, ep: Endpoint, model, prompt):
        try:
            async with self.session.post(ep.url + "/tokenize", json={"model": model, "prompt": prompt},
                                         timeout=aiohttp.ClientTimeout(total=10)) as r:
                if r.status == 200:
                    return (await r.json())["tokens"]
        except RETRYABLE:
            pass
        return None

    # ---------------------------------------------------------------- core
    async def _attempt(self, st: Resumer, ep: Endpoint, path: str):
        """Stream one backend attempt, yielding client chunks; raises if the
        stream ends without ``[DONE]``."""
        req = await st.build(ep)
        base_k = st.k
        ep.inflight += 1
        try:
            async with self.session.post(ep.url + path, json=req) as r:
                st.resp, st.ep = r, ep
                if r.status != 200:
                    payload = await r.read()
                    if r.status >= 500 or r.status in (404, 408, 429) or base_k > 0:
                        raise StreamBroken(f"HTTP {r.status}")
                    raise HTTPPassthrough(r.status, payload, r.content_type)
                loop = asyncio.get_running_loop()
                last = [loop.time()]
                fired = [False]
                dog = None
                started = base_k > 0
                try:
                    while True:
                        if started:
                            if dog is None and self.idle_timeout:
                                dog = asyncio.ensure_future(self._watchdog(r, last, fired, ep.dead))
                            try:
                                line = await r.content.readline()
                            except RETRYABLE:
                                if fired[0]:
                                    raise asyncio.TimeoutError()
                                raise
                            if fired[0]:
                                raise asyncio.TimeoutError()
                            last[0] = loop.time()
                        else:
                            line = await self._wait_first(r.content, ep, getattr(st, "abort_first", None))
                        if not line:
                            raise StreamBroken("EOF before [DONE]")
                        if not line.startswith(b"data:"):
                            continue
                        data = line[5:].strip()
                        if data == b"[DONE]":
                            return
                        obj = _loads(data)
                        if isinstance(obj, dict) and obj.get("error") and not obj.get("choices"):
                            raise StreamBroken(f"backend error: {str(obj['error'])[:200]}")
                        out = st.on_chunk(obj, base_k)
                        started = started or st.k > base_k
                        if out is not None:
                            yield out
                finally:
                    if dog is not None:
                        dog.cancel()
        finally:
            st.resp = None
            ep.inflight -= 1

    async def _watchdog(self, r, last, fired, dead: Optional[asyncio.Event] = None):
        """Close ``r`` after ``idle_timeout`` without a line, or as soon as
        the replica is declared dead, so the pending read fails over."""
        loop = asyncio.get_running_loop()
        dw = asyncio.ensure_future(dead.wait()) if dead is not None else None
        try:
            while True:
                left = last[0] + self.idle_timeout - loop.time()
                if left <= 0 or (dw is not None and dw.done()):
                    fired[0] = True
                    r.close()
                    return
                if dw is not None:
                    await asyncio.wait({dw}, timeout=max(left, 0.01))
                else:
                    await asyncio.sleep(max(left, 0.01))
        finally:
            if dw is not None and not dw.done():
                dw.cancel()

    async def _wait_first(self, content, ep: Endpoint, abort=None):
        """Next line before the first token: no idle limit; ends early only if
        the replica is declared dead or ``abort()`` (a coroutine factory)
        finishes first."""
        read = asyncio.ensure_future(content.readline())
        dead = asyncio.ensure_future(ep.dead.wait())
        waits = {read, dead}
        ab = asyncio.ensure_future(abort()) if abort is not None else None
        if ab is not None:
            waits.add(ab)
        try:
            done, _ = await asyncio.wait(waits, timeout=self.first_token_timeout, return_when=asyncio.FIRST_COMPLETED)
            if read in done:
                return read.result()
            if ab is not None and ab in done:
                raise StreamBroken(f"aborted before first token: {ab.result()}")
            raise StreamBroken("replica died before first token" if done else "first-token timeout")
        finally:
            for t in (dead, ab):
                if t is not None:
                    t.cancel()
            if not read.done():
                read.cancel()

    async def generate(self, kind: str, body: dict):
        """Client chunks of one request (retry / resume inside); the final
        item is the :class:`Resumer` itself."""
        st = self.resumer_cls(self, kind, body)
        self.begin(st)
        try:
            async for c in self._generate(st):
                yield c
        finally:
            self.end(st)

    def begin(self, st: Resumer) -> None:
        """Hook: ``st`` admitted."""

    def end(self, st: Resumer) -> None:
        """Hook: ``st`` finished, failed or was cancelled."""

    async def _generate(self, st: Resumer):
        path = "/v1/chat/completions" if st.chat else "/v1/completions"
        self.stats["requests"] += 1
        tried: List[str] = []
        last_err = "no endpoints"
        while st.attempts < self.max_attempts:
            rem = st.remaining()
            if st.k > 0 and (st.finish is not None or (rem is not None and rem <= 0)):
                # broke after its last token but before [DONE]: complete already
                st.finish = st.finish or "length"
                yield st
                return
            ep = self.pick(st, tried)
            if ep is None:
                break
            st.attempts += 1
            if st.attempts > 1:
                self.stats["resumes" if st.k else "retries"] += 1
            k0 = st.k
            try:
                async for c in self._attempt(st, ep, path):
                    yield c
                yield st
                return
            except HTTPPassthrough:
                raise
            except (StreamBroken, ValueError, KeyError, *RETRYABLE) as e:
                if st.moved:        # planned cut-over: no blame, no attempt used
                    st.moved = False
                    st.attempts -= 1
                    self.stats["moves"] = self.stats.get("moves", 0) + 1
                    continue
                last_err = f"idle > {self.idle_timeout}s" if isinstance(e, asyncio.TimeoutError) \
                    else f"{type(e).__name__}: {e}"
                if getattr(st, "spare_endpoint", False):
                    st.spare_endpoint = False       # not this replica's fault
                elif isinstance(e, asyncio.TimeoutError) and await self._alive(ep):
                    log.info("%s idle but alive: resuming elsewhere without blacklisting", ep.url)
                else:
                    self.pool.mark_bad(ep, last_err)
                tried.append(ep.url)
                if len(tried) >= len(self.pool.order):
                    tried = tried[-1:]
                log.warning("attempt %d on %s failed after %d tokens (%d here): %s", st.attempts, ep.url, st.k,
                            st.k - k0, last_err)
                if not st.can_resume():
                    break
        self.stats["failed"] += 1
        raise UpstreamFailed(last_err, st)

    def pick(self, st: Resumer, tried) -> Optional[Endpoint]:
        """Replica for the next attempt (session-aware routers override)."""
        return self.pool.pick(exclude=tried) or self.pool.pick()

    def move(self, st: Resumer) -> bool:
        """Cut ``st`` over: close its backend stream and resume it elsewhere."""
        if st.resp is None or not st.can_resume():
            return False
        st.moved = True
        st.resp.close()
        return True

    # ------------------------------------------------------------ handlers
    async def handle_completions(self, request):
        return await self._handle(request, "completions")

    async def handle_chat(self, request):
        return await self._handle(request, "chat")

    async def _handle(self, request, kind: str):
        body = await request.json()
        gen = self.generate(kind, body)
        if body.get("stream"):
            return await self._stream(request, gen)
        return await self._aggregate(gen, kind)

    async def _stream(self, request, gen):
        resp = None
        try:
            async for c in gen:
                if isinstance(c, Resumer):
                    if resp is None:
                        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream"})
                        await resp.prepare(request)
                    if c.client_usage:
                        await resp.write(_sse({"id": c.rid, "object": _obj(c.chat), "created": c.created,
                                               "model": c.model, "choices": [], "usage": c.usage()}))
                    await resp.write(b"data: [DONE]\n\n")
                    break
                if resp is None:
                    resp = web.StreamResponse(headers={"Content-Type": "text/event-stream",
                                                       "Cache-Control": "no-cache"})
                    await resp.prepare(request)
                await resp.write(_sse(c))
        except HTTPPassthrough as e:
            if resp is None:
                return web.Response(status=e.status, body=e.payload, content_type=e.ctype)
            raise
        except UpstreamFailed as e:
            if resp is None:
                return web.json_response({"error": {"message": f"all replicas failed: {e}",
                                                    "type": "upstream_failed"}}, status=502)
            await resp.write(_sse({"error": {"message": f"stream lost after {e.st.k} tokens: {e}",
                                             "type": "upstream_failed"}}))
            await resp.write(b"data: [DONE]\n\n")
        await resp.write_eof()
        return resp

    async def _aggregate(self, gen, kind: str):
        text, lps, st = [], [], None
        try:
            async for c in gen:
                if isinstance(c, Resumer):
                    st = c
                    break
                ch = c["choices"][0]
                text.append(((ch.get("delta") or {}).get("content") or "") if kind == "chat" else (ch.get("text") or ""))
                if ch.get("logprobs"):
                    lps.append(ch["logprobs"])
        except HTTPPassthrough as e:
            return web.Response(status=e.status, body=e.payload, content_type=e.ctype)
        except UpstreamFailed as e:
            return web.json_response({"error": {"message": f"all replicas failed: {e}", "type": "upstream_failed"}},
                                     status=502)
        content = "".join(text)
        lp = _merge_lp(lps, kind == "chat")
        if kind == "chat":
            choice = {"index": 0, "message": {"role": "assistant", "content": content}, "logprobs": lp,
                      "finish_reason": st.finish, "stop_reason": st.stop_reason}
        else:
            choice = {"index": 0, "text": content, "logprobs": lp, "finish_reason": st.finish,
                      "stop_reason": st.stop_reason}
        return web.json_response({"id": st.rid, "object": "chat.completion" if kind == "chat" else "text_completion",
                                  "created": st.created, "model": st.model, "choices": [choice], "usage": st.usage()})

    async def handle_models(self, request):
        for _ in range(len(self.pool.order) or 1):
            ep = self.pool.pick()
            if ep is None:
                break
            try:
                async with self.session.get(ep.url + "/v1/models", timeout=aiohttp.ClientTimeout(total=5)) as r:
                    return web.Response(status=r.status, body=await r.read(), content_type=r.content_type)
            except RETRYABLE as e:
                self.pool.mark_bad(ep, f"models: {e}")
        return web.json_response({"error": "no healthy replica"}, status=502)

    async def handle_health(self, request):
        now = time.monotonic()
        ok = any(self.pool.eps[u].healthy(now) for u in self.pool.order)
        return web.json_response({"healthy": ok}, status=200 if ok else 503)

    async def handle_stats(self, request):
        now = time.monotonic()
        eps = [{"url": u, "healthy": self.pool.eps[u].healthy(now), "inflight": self.pool.eps[u].inflight}
               for u in self.pool.order]
        return web.json_response({**self.stats, "endpoints": eps})


def _obj(chat: bool) -> str:
    return "chat.completion.chunk" if chat else "text_completion"


def _merge_lp(lps, chat: bool):
    if not lps:
        return None
    if chat:
        return {"content": [x for lp in lps for x in lp.get("content") or []]}
    out = {"tokens": [], "token_logprobs": [], "top_logprobs": [], "text_offset": []}
    for lp in lps:
        for k in out:
            out[k].extend(lp.get(k) or [])
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description="Resume proxy for OpenAI-API replicas")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=5199)
    ap.add_argument("--endpoints", default="", help="comma-separated replica base URLs")
    ap.add_argument("--endpoints-file", default=None, help="one URL per line; removal = dead")
    ap.add_argument("--reload-interval", type=float, default=1.0)
    ap.add_argument("--idle-timeout", type=float, default=2.5)
    ap.add_argument("--first-token-timeout", type=float, default=None)
    ap.add_argument("--connect-timeout", type=float, default=2.0)
    ap.add_argument("--max-attempts", type=int, default=4)
    ap.add_argument("--blacklist-s", type=float, default=5.0)
    ap.add_argument("--probe-interval", type=float, default=1.0, help="0 disables probing")
    ap.add_argument("--no-token-ids", action="store_true", help="resume completions from text")
    ap.add_argument("--log-level", default="INFO")
    a = ap.parse_args()
    logging.basicConfig(level=a.log_level, format="%(asctime)s %(name)s %(levelname)s %(message)s")
    pool = Pool([u for u in a.endpoints.split(",") if u], a.endpoints_file, a.blacklist_s)
    proxy = Proxy(pool, a.idle_timeout, a.connect_timeout, a.max_attempts, a.probe_interval, not a.no_token_ids,
                  a.first_token_timeout)
    proxy.reload_interval = a.reload_interval
    web.run_app(proxy.app(), host=a.host, port=a.port, access_log=None)


if __name__ == "__main__":
    main()

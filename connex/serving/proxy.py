"""Resume proxy: an OpenAI-API front that hides replica deaths from clients.

Replicas
    come from ``--endpoints`` and/or an endpoints file (re-read every
    ``--reload-interval`` s; a URL removed from the file counts as dead).  A
    prober GETs ``/v1/models`` on fresh connections; two failed probes in a
    row, a refused connect or a broken stream blacklist a replica for
    ``--blacklist-s``.  Requests go to the least loaded healthy replica.

One client request is a :class:`Resumer`: the body of the next backend
attempt, and a ledger of what the client has been sent (text, token ids,
completion-token count, id / created / model of the first attempt).  Every
attempt streams, whatever the client asked for; :class:`_Lines` reads the
backend's lines under two regimes:

* **before the first token** there is no idle limit -- a long prefill is
  never cut; the wait ends only when the replica is declared dead, an
  optional first-token cap passes, or the request's own guard fires (the
  PD router's SGLang prefill);
* **after a token**, ``--idle-timeout`` without a line, or the replica's
  death, ends the attempt.

A failed attempt before the first token is retried elsewhere; after k
tokens the request *resumes* elsewhere: completions from token ids (prompt
ids + generated ids: the proxy asks for ``return_token_ids`` / id logprobs
and strips what the client did not ask for), chat through
``continue_final_message``; ``max_tokens`` / ``min_tokens`` shrink by k.  The
client sees one stream with one ``id`` and a usage block counting the
original prompt and every completion token.  :meth:`Proxy.move` cuts a
request over on purpose (planned migration; no blame, no attempt used).

Behavioural parity: ``connex/serving/proxy.py:84-764`` of the reference
(routes, flags, resume semantics); the structure here is this module's own.

    python -m connex.serving.proxy --port 5199 --endpoints http://a:5100,http://b:5101
"""
from __future__ import annotations

import argparse
import asyncio
import json
import logging
import time
from typing import AsyncIterator, Callable, Dict, List, Optional

import aiohttp
from aiohttp import web

log = logging.getLogger("connex.proxy")

RETRYABLE = (aiohttp.ClientError, asyncio.TimeoutError, ConnectionError, OSError)
_ID_PREFIX = "token_id:"


def _sse(obj) -> bytes:
    return b"data: " + json.dumps(obj, separators=(",", ":")).encode() + b"\n\n"


class StreamBroken(Exception):
    """The backend stream ended or failed before ``[DONE]``."""


class HTTPPassthrough(Exception):
    """A client error from the backend (4xx before any token): forwarded as is."""

    def __init__(self, status, payload, ctype):
        super().__init__(f"HTTP {status}")
        self.status, self.payload, self.ctype = status, payload, ctype or "application/json"


class UpstreamFailed(Exception):
    def __init__(self, msg, st):
        super().__init__(msg)
        self.st = st


# ================================================================ replicas
class Endpoint:
    """One replica: health (blacklisted until ``bad_until``), load, and an
    event that is set while it is blacklisted (waiters on it wake up)."""

    __slots__ = ("url", "bad_until", "inflight", "dead")

    def __init__(self, url: str):
        self.url = url.rstrip("/")
        self.bad_until = 0.0
        self.inflight = 0
        self.dead = asyncio.Event()

    def healthy(self, now: float) -> bool:
        return now >= self.bad_until


def _clean(urls) -> List[str]:
    return [u.strip().rstrip("/") for u in urls if u.strip()]


class Pool:
    def __init__(self, urls=(), endpoints_file: Optional[str] = None, blacklist_s: float = 5.0):
        self.eps: Dict[str, Endpoint] = {}
        self.order: List[str] = []
        self.file = endpoints_file
        self.blacklist_s = blacklist_s
        self._turn = 0
        self.set_urls(urls)

    def set_urls(self, urls) -> None:
        urls = _clean(urls)
        for u in urls:
            if u not in self.eps:
                self.eps[u] = Endpoint(u)
        self.order = urls

    def _file_urls(self) -> Optional[List[str]]:
        try:
            with open(self.file) as f:
                return _clean(f)
        except OSError:
            return None

    def reload(self) -> None:
        """Re-read the endpoints file; a URL that left it is dead now."""
        listed = self._file_urls() if self.file else None
        if not listed:
            return
        removed = [u for u in self.order if u not in listed]
        self.set_urls(listed)
        for u in removed:
            self.mark_bad(self.eps[u], "removed from endpoints file")

    def mark_bad(self, ep: Endpoint, why: str = "") -> None:
        now = time.monotonic()
        if ep.healthy(now):
            log.warning("blacklisting %s for %.1fs: %s", ep.url, self.blacklist_s, why)
        ep.bad_until = now + self.blacklist_s
        ep.dead.set()

    def mark_good(self, ep: Endpoint) -> None:
        if ep.bad_until:
            ep.bad_until = 0.0
            ep.dead = asyncio.Event()

    def pick(self, exclude=()) -> Optional[Endpoint]:
        """The least loaded healthy replica outside ``exclude`` (ties broken by
        rotation); with none healthy, the one whose blacklist ends first."""
        options = [self.eps[u] for u in self.order if u not in exclude]
        if not options:
            return None
        now = time.monotonic()
        healthy = [e for e in options if e.healthy(now)]
        if not healthy:
            return min(options, key=lambda e: e.bad_until)
        for e in healthy:
            if e.bad_until:              # its blacklist lapsed without a probe: re-arm it
                self.mark_good(e)
        self._turn += 1
        start = self._turn % len(healthy)
        rotated = healthy[start:] + healthy[:start]
        return min(rotated, key=lambda e: e.inflight)


# ================================================================ requests
def _ids_in_logprobs(lp, chat: bool) -> Optional[List[int]]:
    """Token ids carried as ``token_id:<n>`` strings in a logprobs block."""
    if not lp:
        return None
    names = [c.get("token") for c in lp.get("content") or []] if chat else lp.get("tokens")
    if not names or not all(isinstance(n, str) and n.startswith(_ID_PREFIX) for n in names):
        return None
    return [int(n[len(_ID_PREFIX):]) for n in names]


class Resumer:
    """One client request across its backend attempts.

    What the client has received so far: ``text`` (pieces), ``ids`` (when
    the backend reports token ids), ``k`` (completion tokens), the id /
    created / model of the first attempt, ``finish`` / ``stop_reason``.
    ``build(ep)`` turns that into the body of the next attempt;
    ``on_chunk`` accounts one backend chunk and rewrites it for the client."""

    def __init__(self, proxy: "Proxy", kind: str, body: dict):
        self.p = proxy
        self.kind = kind
        self.chat = kind == "chat"
        self.body = body
        so = body.get("stream_options") or {}
        self.client_usage = bool(so.get("include_usage"))
        self.client_cont_usage = bool(so.get("continuous_usage_stats"))
        prompt = body.get("prompt")
        one_choice = body.get("n") in (None, 1) and body.get("best_of") in (None, 1)
        single_prompt = isinstance(prompt, str) or (isinstance(prompt, list) and bool(prompt)
                                                    and isinstance(prompt[0], int))
        self.resumable = one_choice and (self.chat or single_prompt)
        lp = body.get("logprobs")
        self.client_lp = lp is not None and lp is not False     # logprobs=0 asks for them too
        self.use_ids = (self.resumable and not self.chat and proxy.token_ids
                        and (not self.client_lp or bool(body.get("return_tokens_as_token_ids"))))
        self.inject_lp = self.use_ids and not self.client_lp
        self.prompt_ids: Optional[List[int]] = prompt if isinstance(prompt, list) else None
        self.model = body.get("model")
        # the ledger
        self.ids: List[int] = []
        self.text: List[str] = []
        self.k = 0
        self.prompt_tokens = None
        self.rid = self.created = None
        self.finish = self.stop_reason = None
        self.sent_role = False
        # the current attempt
        self.attempts = 0
        self.resp = None
        self.ep: Optional[Endpoint] = None
        self.moved = False

    # ------------------------------------------------------------ next body
    def _common(self) -> dict:
        b = dict(self.body)
        b["stream"] = True
        b["stream_options"] = {"include_usage": True, "continuous_usage_stats": True}
        if self.inject_lp:
            b["logprobs"] = True if self.chat else 0
            b["return_tokens_as_token_ids"] = True
        if self.use_ids:
            b["return_token_ids"] = True
        return b

    def _shrink(self, b: dict) -> None:
        for key in ("max_tokens", "max_completion_tokens"):
            if b.get(key) is not None:
                b[key] -= self.k
        if b.get("min_tokens"):
            b["min_tokens"] = max(0, b["min_tokens"] - self.k)

    def _chat_continuation(self, b: dict) -> dict:
        done = "".join(self.text)
        msgs = [dict(m) for m in b["messages"]]
        if b.get("continue_final_message") and msgs and msgs[-1].get("role") == "assistant":
            msgs[-1]["content"] = (msgs[-1].get("content") or "") + done
        else:
            msgs.append({"role": "assistant", "content": done})
        b.update(messages=msgs, add_generation_prompt=False, continue_final_message=True)
        return b

    async def _completion_continuation(self, b: dict, ep: Endpoint) -> dict:
        b["echo"] = False
        if self.use_ids and len(self.ids) == self.k:
            if self.prompt_ids is None:
                self.prompt_ids = await self.p.tokenize(ep, self.model, self.body["prompt"])
            if self.prompt_ids is not None:
                b["prompt"] = list(self.prompt_ids) + self.ids
                return b
        if isinstance(b["prompt"], str):
            b["prompt"] += "".join(self.text)
            return b
        raise StreamBroken("cannot resume a token-id prompt without the generated ids")

    async def build(self, ep: Endpoint) -> dict:
        """The backend body of the next attempt (on ``ep``)."""
        b = self._common()
        if self.k == 0:
            return b
        self._shrink(b)
        if self.chat:
            return self._chat_continuation(b)
        return await self._completion_continuation(b, ep)

    def first_token_guard(self) -> Optional[Callable]:
        """An awaitable factory whose completion before the first token ends
        the attempt (its result is the reason); None for no guard."""
        return None

    def can_resume(self) -> bool:
        return self.k == 0 or self.resumable

    def remaining(self):
        m = self.body.get("max_tokens")
        if m is None:
            m = self.body.get("max_completion_tokens")
        return None if m is None else m - self.k

    def complete_already(self) -> bool:
        """The stream broke after its last token (before ``[DONE]``)."""
        rem = self.remaining()
        return self.k > 0 and (self.finish is not None or (rem is not None and rem <= 0))

    # -------------------------------------------------------------- ledger
    def _count(self, ch: dict, usage: Optional[dict], base_k: int, piece: str) -> None:
        ids = ch.get("token_ids")
        if not ids and self.use_ids:
            ids = _ids_in_logprobs(ch.get("logprobs"), self.chat)
        if usage and usage.get("completion_tokens") is not None:
            self.k = base_k + usage["completion_tokens"]
        elif ids:
            self.k += len(ids)
        elif piece:
            self.k += 1
        if self.use_ids:
            self.ids.extend(ids or [])
            if len(self.ids) != self.k:
                self.use_ids = False            # lost count: resume from text instead

    def _for_client(self, c: dict, ch: dict) -> dict:
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

    def on_chunk(self, c: dict, base_k: int) -> Optional[dict]:
        """Account one backend chunk; returns the chunk for the client, or None."""
        usage = c.get("usage")
        choices = c.get("choices") or []
        if usage and base_k == 0 and self.prompt_tokens is None:
            self.prompt_tokens = usage.get("prompt_tokens")
        if not choices:                         # a usage-only chunk: ours replaces it at the end
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
                    return None                 # the role preamble of a retried / resumed stream
                self.sent_role = True
        else:
            piece = ch.get("text") or ""
        self._count(ch, usage, base_k, piece)
        self.text.append(piece)
        if ch.get("finish_reason") is not None:
            self.finish, self.stop_reason = ch["finish_reason"], ch.get("stop_reason")
        return self._for_client(c, ch)

    def usage(self) -> dict:
        pt = self.prompt_tokens
        if pt is None and self.prompt_ids is not None:
            pt = len(self.prompt_ids)
        return {"prompt_tokens": pt, "completion_tokens": self.k, "total_tokens": (pt or 0) + self.k}


class _Lines:
    """The lines of one backend response under the proxy's timing rules."""

    def __init__(self, resp, ep: Endpoint, idle_timeout: Optional[float], first_token_timeout: Optional[float],
                 guard: Optional[Callable]):
        self.resp, self.ep = resp, ep
        self.idle, self.first_cap = idle_timeout, first_token_timeout
        self.guard_task = asyncio.ensure_future(guard()) if guard is not None else None

    async def next(self, started: bool) -> bytes:
        read = asyncio.ensure_future(self.resp.content.readline())
        death = asyncio.ensure_future(self.ep.dead.wait())
        waits = {read, death}
        if not started and self.guard_task is not None:
            waits.add(self.guard_task)
        limit = self.idle if started else self.first_cap
        try:
            done, _ = await asyncio.wait(waits, timeout=limit or None, return_when=asyncio.FIRST_COMPLETED)
        finally:
            death.cancel()
        if read in done:
            return read.result()
        read.cancel()
        self.resp.close()
        if self.guard_task is not None and self.guard_task in done:
            raise StreamBroken(f"aborted before first token: {self.guard_task.result()}")
        if death in done:
            raise StreamBroken("replica died" + ("" if started else " before first token"))
        if started:
            raise asyncio.TimeoutError()        # idle: the caller checks whether the replica lives
        raise StreamBroken("first-token timeout")

    def close(self) -> None:
        if self.guard_task is not None and not self.guard_task.done():
            self.guard_task.cancel()


# ================================================================== proxy
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
        self.stats = {"requests": 0, "retries": 0, "resumes": 0, "failed": 0, "moves": 0}
        self._bg: List[asyncio.Task] = []

    # -------------------------------------------------------------- lifecycle
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
            self._background(self._every(self.reload_interval, self.pool.reload))
        if self.probe_interval:
            self._background(self._probe_loop())

    def _background(self, coro) -> None:
        self._bg.append(asyncio.create_task(coro))

    async def _cleanup(self, app=None):
        for t in self._bg:
            t.cancel()
        await self.session.close()
        await self.probe_session.close()

    async def _every(self, period: float, fn) -> None:
        while True:
            await asyncio.sleep(period)
            fn()

    # ---------------------------------------------------------------- probes
    def _probe_targets(self) -> List[tuple]:
        """(endpoint, its pool) of every listed replica."""
        return [(e, self.pool) for e in list(self.pool.eps.values()) if e.url in self.pool.order]

    async def _probe_loop(self):
        while True:
            await asyncio.sleep(self.probe_interval)
            await asyncio.gather(*(self._probe(e, p) for e, p in self._probe_targets()), return_exceptions=True)

    async def _alive(self, ep: Endpoint, timeout: float = 2.0) -> bool:
        try:
            async with self.probe_session.get(ep.url + "/v1/models",
                                              timeout=aiohttp.ClientTimeout(total=timeout)) as r:
                return r.status == 200
        except RETRYABLE:
            return False

    async def _probe(self, ep: Endpoint, pool: Optional[Pool] = None) -> None:
        # two failures in a row: a busy but alive server keeps its prefills
        pool = pool or self.pool
        if await self._alive(ep) or await self._alive(ep):
            pool.mark_good(ep)
        else:
            pool.mark_bad(ep, "probe failed twice")

    async def tokenize(self, ep: Endpoint, model, prompt):
        try:
            async with self.session.post(ep.url + "/tokenize", json={"model": model, "prompt": prompt},
                                         timeout=aiohttp.ClientTimeout(total=10)) as r:
                if r.status == 200:
                    return (await r.json())["tokens"]
        except RETRYABLE:
            pass
        return None

    # ------------------------------------------------------------- attempts
    @staticmethod
    def _path(st: Resumer) -> str:
        return "/v1/chat/completions" if st.chat else "/v1/completions"

    async def _attempt(self, st: Resumer, ep: Endpoint) -> AsyncIterator[dict]:
        """Stream one backend attempt, yielding client chunks; returns at
        ``[DONE]``, raises otherwise."""
        body = await st.build(ep)
        base_k = st.k
        ep.inflight += 1
        lines = None
        try:
            async with self.session.post(ep.url + self._path(st), json=body) as r:
                st.resp, st.ep = r, ep
                if r.status != 200:
                    payload = await r.read()
                    if r.status >= 500 or r.status in (404, 408, 429) or base_k > 0:
                        raise StreamBroken(f"HTTP {r.status}")
                    raise HTTPPassthrough(r.status, payload, r.content_type)
                lines = _Lines(r, ep, self.idle_timeout, self.first_token_timeout, st.first_token_guard())
                while True:
                    line = await lines.next(started=st.k > base_k or base_k > 0)
                    if not line:
                        raise StreamBroken("EOF before [DONE]")
                    if not line.startswith(b"data:"):
                        continue
                    data = line[5:].strip()
                    if data == b"[DONE]":
                        return
                    obj = json.loads(data)
                    if isinstance(obj, dict) and obj.get("error") and not obj.get("choices"):
                        raise StreamBroken(f"backend error: {str(obj['error'])[:200]}")
                    out = st.on_chunk(obj, base_k)
                    if out is not None:
                        yield out
        finally:
            if lines is not None:
                lines.close()
            st.resp = None
            ep.inflight -= 1

    async def on_attempt_failed(self, st: Resumer, ep: Endpoint, err: BaseException, produced: int) -> bool:
        """Whether to blacklist ``ep`` after a failed attempt that produced
        ``produced`` tokens.  An idle stream on a replica that still answers
        is not its death."""
        if isinstance(err, asyncio.TimeoutError) and await self._alive(ep):
            log.info("%s idle but alive: resuming elsewhere without blacklisting", ep.url)
            return False
        return True

    # ------------------------------------------------------------- requests
    def make_request(self, kind: str, body: dict) -> Resumer:
        return self.resumer_cls(self, kind, body)

    async def generate(self, kind: str, body: dict):
        """Client chunks of one request (retry / resume inside); the final
        item is the :class:`Resumer` itself."""
        st = self.make_request(kind, body)
        self.begin(st)
        try:
            async for c in self._drive(st):
                yield c
        finally:
            self.end(st)

    def begin(self, st: Resumer) -> None:
        """Hook: ``st`` admitted."""

    def end(self, st: Resumer) -> None:
        """Hook: ``st`` finished, failed or was cancelled."""

    def pick(self, st: Resumer, tried) -> Optional[Endpoint]:
        """Replica for the next attempt (session-aware routers override)."""
        return self.pool.pick(exclude=tried) or self.pool.pick()

    async def _drive(self, st: Resumer):
        self.stats["requests"] += 1
        tried: List[str] = []
        reason = "no endpoints"
        while st.attempts < self.max_attempts:
            if st.complete_already():
                st.finish = st.finish or "length"
                yield st
                return
            ep = self.pick(st, tried)
            if ep is None:
                break
            st.attempts += 1
            if st.attempts > 1:
                self.stats["resumes" if st.k else "retries"] += 1
            k_before = st.k
            try:
                async for c in self._attempt(st, ep):
                    yield c
                yield st
                return
            except HTTPPassthrough:
                raise
            except (StreamBroken, ValueError, KeyError, *RETRYABLE) as e:
                if st.moved:                    # planned cut-over: no blame, no attempt used
                    st.moved = False
                    st.attempts -= 1
                    self.stats["moves"] += 1
                    continue
                reason = f"idle > {self.idle_timeout}s" if isinstance(e, asyncio.TimeoutError) \
                    else f"{type(e).__name__}: {e}"
                if await self.on_attempt_failed(st, ep, e, st.k - k_before):
                    self.pool.mark_bad(ep, reason)
                tried.append(ep.url)
                if len(tried) >= len(self.pool.order):
                    tried = tried[-1:]
                log.warning("attempt %d on %s failed after %d tokens (%d here): %s", st.attempts, ep.url, st.k,
                            st.k - k_before, reason)
                if not st.can_resume():
                    break
        self.stats["failed"] += 1
        raise UpstreamFailed(reason, st)

    def move(self, st: Resumer) -> bool:
        """Cut ``st`` over: close its backend stream and resume it elsewhere."""
        if st.resp is None or not st.can_resume():
            return False
        st.moved = True
        st.resp.close()
        return True

    # -------------------------------------------------------------- handlers
    async def handle_completions(self, request):
        return await self._handle(request, "completions")

    async def handle_chat(self, request):
        return await self._handle(request, "chat")

    async def _handle(self, request, kind: str):
        body = await request.json()
        return await self.respond(request, kind, body)

    async def respond(self, request, kind: str, body: dict):
        gen = self.generate(kind, body)
        if body.get("stream"):
            return await self._stream(request, gen)
        return await self._aggregate(gen, kind)

    async def _stream(self, request, gen):
        resp = None

        async def opened():
            nonlocal resp
            if resp is None:
                resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
                await resp.prepare(request)
            return resp
        try:
            async for c in gen:
                if isinstance(c, Resumer):
                    out = await opened()
                    if c.client_usage:
                        await out.write(_sse({"id": c.rid, "object": _obj(c.chat), "created": c.created,
                                              "model": c.model, "choices": [], "usage": c.usage()}))
                    await out.write(b"data: [DONE]\n\n")
                    break
                await (await opened()).write(_sse(c))
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
        pieces, lps, st = [], [], None
        try:
            async for c in gen:
                if isinstance(c, Resumer):
                    st = c
                    break
                ch = c["choices"][0]
                pieces.append(((ch.get("delta") or {}).get("content") or "") if kind == "chat"
                              else (ch.get("text") or ""))
                if ch.get("logprobs"):
                    lps.append(ch["logprobs"])
        except HTTPPassthrough as e:
            return web.Response(status=e.status, body=e.payload, content_type=e.ctype)
        except UpstreamFailed as e:
            return web.json_response({"error": {"message": f"all replicas failed: {e}", "type": "upstream_failed"}},
                                     status=502)
        content = "".join(pieces)
        lp = _merge_lp(lps, kind == "chat")
        base = {"index": 0, "logprobs": lp, "finish_reason": st.finish, "stop_reason": st.stop_reason}
        choice = {**base, "message": {"role": "assistant", "content": content}} if kind == "chat" \
            else {**base, "text": content}
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
    """One logprobs block from the per-chunk blocks."""
    if not lps:
        return None
    if chat:
        return {"content": [x for lp in lps for x in lp.get("content") or []]}
    keys = ("tokens", "token_logprobs", "top_logprobs", "text_offset")
    return {k: [x for lp in lps for x in (lp.get(k) or [])] for k in keys}


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

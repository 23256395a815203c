"""Deterministic fake OpenAI-API servers for CPU tests of the serving layer.

The "model" (:func:`next_token`) is greedy and remembers only two tokens:
the next id is a pure function of the last two ids, so generating from
``prompt + partial output`` continues an interrupted stream exactly.  Id
``i`` is the word ``t{i}`` (text ``" t{i}"``).  The server speaks the API
subset the resume proxy and the PD router use: ``/v1/completions`` and
``/v1/chat/completions`` (streamed or not, ``stream_options``, id logprobs,
``return_token_ids``, id prompts, chat ``continue_final_message``),
``/tokenize``, ``/v1/models`` and ``/health``.

Fault injection: ``fail = ("reset", k)`` drops the connection after k
tokens, ``("stall", k)`` stops sending after k tokens with the socket open,
``("http500", 0)`` answers 500; ``fail_count`` bounds how many requests fail.

:class:`FakePDBackend` and :class:`FakeSGLangPDBackend` add the prefill /
decode hand-off semantics of vLLM's ``kv_transfer_params`` and SGLang's
``bootstrap_room``.  Behavioural parity: ``connex/serving/fake_backend.py``
of the reference (same routes, fault knobs and PD semantics).

    python -m connex.serving.fake_backend --port 5100
"""
from __future__ import annotations

import argparse
import asyncio
import json
import time
from dataclasses import dataclass
from typing import AsyncIterator, List, Optional

from aiohttp import web

VOCAB = 1000
BOS = 1
EOT = 4
CHAT_HEADER = [2, 3]


def next_token(ids, vocab: int = VOCAB) -> int:
    """The greedy next id after ``ids`` (a function of the last two only)."""
    last = ids[-1] if len(ids) > 0 else 0
    before = ids[-2] if len(ids) > 1 else 0
    return (last * 131 + before * 29 + 7) % (vocab - 16) + 16


def tokenize(text: str, add_bos: bool = True) -> List[int]:
    """``t<i>`` words are id ``i``; any other word hashes to an id."""
    ids = [BOS] if add_bos else []
    for word in text.split():
        numeric = word[:1] == "t" and word[1:].isdigit()
        ids.append(int(word[1:]) % VOCAB if numeric else sum(word.encode()) % VOCAB)
    return ids


def detok(t: int) -> str:
    return f" t{t}"


def chat_ids(messages, add_generation_prompt=True, continue_final=False) -> List[int]:
    ids = [BOS]
    last = len(messages) - 1
    for i, m in enumerate(messages):
        ids += CHAT_HEADER + tokenize(m.get("content") or "", add_bos=False)
        if i != last or not continue_final:
            ids.append(EOT)
    if add_generation_prompt and not continue_final:
        ids += CHAT_HEADER
    return ids


def continuation(ids, n: int) -> List[int]:
    seq, out = list(ids), []
    for _ in range(n):
        seq.append(next_token(seq))
        out.append(seq[-1])
    return out


def reference(prompt, max_tokens: int):
    """Uninterrupted greedy completion: (ids, text)."""
    out = continuation(tokenize(prompt) if isinstance(prompt, str) else list(prompt), max_tokens)
    return out, "".join(detok(t) for t in out)


@dataclass
class _Reply:
    """What one generation request asked for."""

    rid: str
    chat: bool
    prompt_len: int
    tokens: List[int]
    logprobs: bool
    ids_as_text: bool
    token_ids: bool
    usage_each: bool
    usage_end: bool

    @property
    def kind(self) -> str:
        return "chat.completion.chunk" if self.chat else "text_completion"

    def usage(self, k: int) -> dict:
        return {"prompt_tokens": self.prompt_len, "completion_tokens": k, "total_tokens": self.prompt_len + k}

    def _logprob(self, t: int) -> dict:
        shown = f"token_id:{t}" if self.ids_as_text else detok(t)
        if self.chat:
            return {"content": [{"token": shown, "logprob": -0.25, "top_logprobs": []}]}
        return {"tokens": [shown], "token_logprobs": [-0.25], "top_logprobs": None, "text_offset": [0]}

    def chunk(self, k: int, model: str, created: int) -> dict:
        t = self.tokens[k]
        fin = "length" if k == len(self.tokens) - 1 else None
        lp = self._logprob(t) if self.logprobs else None
        if self.chat:
            choice = {"index": 0, "delta": {"content": detok(t)}, "logprobs": lp, "finish_reason": fin}
        else:
            choice = {"index": 0, "text": detok(t), "logprobs": lp, "finish_reason": fin, "stop_reason": None}
        if self.token_ids:
            choice["token_ids"] = [t]
        obj = {"id": self.rid, "object": self.kind, "created": created, "model": model, "choices": [choice]}
        if self.usage_each:
            obj["usage"] = self.usage(k + 1)
        return obj

    def whole(self, model: str, created: int) -> dict:
        text = "".join(detok(t) for t in self.tokens)
        if self.chat:
            choice = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": "length"}
        else:
            choice = {"index": 0, "text": text, "finish_reason": "length", "logprobs": None}
        return {"id": self.rid, "object": "chat.completion" if self.chat else "text_completion", "created": created,
                "model": model, "choices": [choice], "usage": self.usage(len(self.tokens))}


class FakeBackend:
    def __init__(self, tpot_ms: float = 0.0, ttft_ms: float = 0.0, model: str = "fake", stamp: bool = False):
        self.tpot = tpot_ms / 1000
        self.ttft = ttft_ms / 1000
        self.model = model
        self.stamp = stamp
        self.fail = None
        self.fail_count: Optional[int] = None
        self.requests: List[dict] = []
        self.runner = None
        self.port = None
        self.url = None

    # ---------------------------------------------------------------- faults
    def _take_fail(self):
        """The injected fault for this request, if any (consumes one of ``fail_count``)."""
        if self.fail is None:
            return None
        if self.fail_count is not None:
            if self.fail_count <= 0:
                return None
            self.fail_count -= 1
        return self.fail

    # ---------------------------------------------------------------- server
    def app(self) -> web.Application:
        app = web.Application()
        app.router.add_post("/v1/completions", self._completions)
        app.router.add_post("/v1/chat/completions", self._chat)
        app.router.add_post("/tokenize", self._tokenize)
        app.router.add_get("/v1/models", self._models)
        app.router.add_get("/health", self._models)
        return app

    async def start(self, port: int = 0, host: str = "127.0.0.1") -> str:
        self.runner = web.AppRunner(self.app(), shutdown_timeout=0.1)
        await self.runner.setup()
        site = web.TCPSite(self.runner, host, port)
        await site.start()
        self.port = site._server.sockets[0].getsockname()[1]
        self.url = f"http://{host}:{self.port}"
        return self.url

    async def stop(self):
        if self.runner:
            await self.runner.cleanup()

    async def _models(self, req):
        return web.json_response({"object": "list", "data": [{"id": self.model, "object": "model"}]})

    async def _tokenize(self, req):
        b = await req.json()
        if "messages" in b:
            ids = chat_ids(b["messages"], b.get("add_generation_prompt", True), b.get("continue_final_message", False))
        else:
            ids = tokenize(b["prompt"], b.get("add_special_tokens", True))
        return web.json_response({"tokens": ids, "count": len(ids), "max_model_len": 4096})

    async def _completions(self, req):
        b = await req.json()
        self.requests.append(b)
        prompt = b["prompt"]
        return await self._generate(req, b, list(prompt) if isinstance(prompt, list) else tokenize(prompt), chat=False)

    async def _chat(self, req):
        b = await req.json()
        self.requests.append(b)
        ids = chat_ids(b["messages"], b.get("add_generation_prompt", True), b.get("continue_final_message", False))
        return await self._generate(req, b, ids, chat=True)

    def _plan(self, b: dict, ids, chat: bool) -> _Reply:
        n = b.get("max_tokens") or b.get("max_completion_tokens") or 16
        so = b.get("stream_options") or {}
        want_lp = b.get("logprobs") is not None and b.get("logprobs") is not False    # logprobs=0 asks too
        return _Reply(rid=f"{'chatcmpl' if chat else 'cmpl'}-{len(self.requests)}", chat=chat, prompt_len=len(ids),
                      tokens=continuation(ids, n), logprobs=want_lp,
                      ids_as_text=bool(b.get("return_tokens_as_token_ids")), token_ids=bool(b.get("return_token_ids")),
                      usage_each=bool(so.get("continuous_usage_stats")), usage_end=bool(so.get("include_usage")))

    async def _events(self, reply: _Reply, created: int, fail) -> AsyncIterator[Optional[dict]]:
        """The stream's JSON events in order; None means "drop the connection now"."""
        if self.ttft:
            await asyncio.sleep(self.ttft)
        if fail and fail[0] == "stall" and fail[1] == 0:
            await asyncio.sleep(3600)
        if reply.chat:
            head = {"id": reply.rid, "object": reply.kind, "created": created, "model": self.model,
                    "choices": [{"index": 0, "delta": {"role": "assistant", "content": ""}, "logprobs": None,
                                 "finish_reason": None}]}
            if reply.usage_each:
                head["usage"] = reply.usage(0)
            yield head
        for k in range(len(reply.tokens)):
            if fail and fail[1] == k:
                if fail[0] == "reset":
                    yield None
                    return
                if fail[0] == "stall":
                    await asyncio.sleep(3600)
            obj = reply.chunk(k, self.model, created)
            if self.stamp:
                obj["_t"] = time.time()
            yield obj
            if self.tpot:
                await asyncio.sleep(self.tpot)
        if reply.usage_end:
            yield {"id": reply.rid, "object": reply.kind, "created": created, "model": self.model, "choices": [],
                   "usage": reply.usage(len(reply.tokens))}

    async def _generate(self, req, b, ids, chat: bool):
        fail = self._take_fail()
        if fail and fail[0] == "http500":
            return web.json_response({"error": "injected failure"}, status=500)
        if b.get("max_tokens") is not None and b["max_tokens"] <= 0:
            return web.json_response({"error": "max_tokens must be positive"}, status=400)
        reply = self._plan(b, ids, chat)
        created = int(time.time())
        if not b.get("stream"):
            return web.json_response(reply.whole(self.model, created))
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream"})
        await resp.prepare(req)
        async for ev in self._events(reply, created, fail):
            if ev is None:
                await asyncio.sleep(0.02)           # let the chunks already written leave, then cut
                req.transport.abort()
                return resp
            await resp.write(b"data: " + json.dumps(ev).encode() + b"\n\n")
        await resp.write(b"data: [DONE]\n\n")
        return resp


class _PDRole(FakeBackend):
    """A fake PD instance: ``alive`` follows start / stop."""

    def __init__(self, role: str, **kw):
        super().__init__(**kw)
        self.role = role
        self.alive = True
        self.prefills = 0

    async def start(self, port=0, host="127.0.0.1"):
        url = await super().start(port, host)
        self.alive = True
        return url

    async def stop(self):
        self.alive = False
        await super().stop()


class FakePDBackend(_PDRole):
    """Fake prefill (``role="prefill"``) or decode instance.  The instances of
    one deployment share ``kv`` (transfer id -> held prompt ids and owner) in
    place of the KV connector: a prefill with ``do_remote_decode`` holds its
    prompt and returns ``kv_transfer_params``; a decode with
    ``do_remote_prefill`` takes the hold and answers 500 if it is gone, its
    owner is down, or the held ids are not the prompt's prefix (wrong KV)."""

    def __init__(self, role: str, kv: dict, **kw):
        super().__init__(role, **kw)
        self.kv = kv
        self.pulls = 0

    async def _prefill(self, req, p: dict, ids):
        fail = self._take_fail()
        if fail and fail[0] == "http500":
            return web.json_response({"error": "injected failure"}, status=500)
        if fail and fail[0] in ("reset", "stall"):
            if fail[0] == "stall":
                await asyncio.sleep(3600)
            req.transport.abort()
            return web.Response()
        self.prefills += 1
        tid = p["transfer_id"]
        self.kv[tid] = {"ids": list(ids), "owner": self}
        return web.json_response({
            "id": "cmpl-prefill", "object": "text_completion", "created": int(time.time()), "model": self.model,
            "choices": [{"index": 0, "text": detok(next_token(ids)), "finish_reason": "length"}],
            "usage": {"prompt_tokens": len(ids), "completion_tokens": 1, "total_tokens": len(ids) + 1},
            "kv_transfer_params": {"do_remote_prefill": True, "do_remote_decode": False, "transfer_id": tid,
                                   "remote_ctrl": self.url, "remote_num_tokens": len(ids)}})

    def _kv_ok(self, p: dict, ids) -> bool:
        held = self.kv.get(p.get("transfer_id"))
        n = p.get("remote_num_tokens", 0)
        return held is not None and held["owner"].alive and len(held["ids"]) == n and held["ids"] == ids[:n]

    async def _generate(self, req, b, ids, chat):
        p = b.get("kv_transfer_params") or {}
        if self.role == "prefill" and p.get("do_remote_decode"):
            return await self._prefill(req, p, ids)
        if self.role == "decode":
            if not p.get("do_remote_prefill"):
                return web.json_response({"error": "decode instance needs kv_transfer_params"}, status=400)
            if not self._kv_ok(p, ids):
                return web.json_response({"error": "KV load failed"}, status=500)
            self.pulls += 1
        return await super()._generate(req, b, ids, chat)


class FakeSGLangPDBackend(_PDRole):
    """Fake SGLang PD instance: prefill and decode receive the same request
    with a ``bootstrap_room``; the decode waits up to ``wait_s`` for the
    prefill to publish the room in the shared ``rooms`` and fails when it
    does not, or when that prefill is down."""

    def __init__(self, role: str, rooms: dict, wait_s: float = 2.0, **kw):
        super().__init__(role, **kw)
        self.rooms, self.wait_s = rooms, wait_s

    async def _room(self, room) -> Optional[tuple]:
        end = time.monotonic() + self.wait_s
        while room not in self.rooms:
            if time.monotonic() > end:
                return None
            await asyncio.sleep(0.005)
        return self.rooms[room]

    async def _generate(self, req, b, ids, chat):
        room = b.get("bootstrap_room")
        if room is None:
            return web.json_response({"error": "bootstrap_room required"}, status=400)
        if self.role == "prefill":
            fail = self._take_fail()
            if fail and fail[0] == "http500":
                return web.json_response({"error": "injected failure"}, status=500)
            self.prefills += 1
            self.rooms[room] = (list(ids), self)
            return await super()._generate(req, {**b, "stream": False, "max_tokens": 1}, ids, chat)
        published = await self._room(room)
        if published is None:
            return web.json_response({"error": "KV transfer timed out"}, status=500)
        held, owner = published
        if held != ids or not owner.alive:
            return web.json_response({"error": "KV transfer failed"}, status=500)
        return await super()._generate(req, b, ids, chat)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=5100)
    ap.add_argument("--tpot-ms", type=float, default=0)
    ap.add_argument("--ttft-ms", type=float, default=0)
    ap.add_argument("--stamp", action="store_true")
    a = ap.parse_args()
    web.run_app(FakeBackend(a.tpot_ms, a.ttft_ms, stamp=a.stamp).app(), host=a.host, port=a.port, access_log=None)


if __name__ == "__main__":
    main()

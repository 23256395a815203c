"""Deterministic fake OpenAI-API server for CPU tests of the serving layer
(reference ``connex/serving/fake_backend.py:65-358``).

The model is greedy and memoryless beyond two tokens: the next id is a pure
function of the last two ids, so generating from ``prompt + partial output``
continues an interrupted stream exactly.  Token ``i`` is the word ``t{i}``
(text ``" t{i}"``).  It serves the API subset the proxy and PD router use:
``/v1/completions`` and ``/v1/chat/completions`` (stream / non-stream,
``stream_options``, id logprobs, ``return_token_ids``, id prompts, chat
``continue_final_message``), ``/tokenize`` and ``/v1/models``.

Fault injection: ``fail = ("reset", k)`` aborts the connection after k
tokens, ``("stall", k)`` stops sending after k tokens with the socket open,
``("http500", 0)`` answers 500; ``fail_count`` bounds how many requests fail.

    python -m connex.serving.fake_backend --port 5100
"""
from __future__ import annotations

import argparse
import asyncio
import json
import time

from aiohttp import web

VOCAB = 1000
BOS = 1
EOT = 4
CHAT_HEADER = [2, 3]


def tokenize(text: str, add_bos: bool = True):
    ids = [BOS] if add_bos else []
    for w in text.split():
        if w.startswith("t") and w[1:].isdigit():
            ids.append(int(w[1:]) % VOCAB)
        else:
            ids.append(sum(w.encode()) % VOCAB)
    return ids


def next_token(ids) -> int:
    a = ids[-1] if ids else 0
    b = ids[-2] if len(ids) > 1 else 0
    return (a * 37 + b * 11 + 5) % (VOCAB - 16) + 16


def detok(t: int) -> str:
    return f" t{t}"


def chat_ids(messages, add_generation_prompt=True, continue_final=False):
    ids = [BOS]
    for i, m in enumerate(messages):
        ids += CHAT_HEADER + tokenize(m.get("content") or "", add_bos=False)
        if not (i == len(messages) - 1 and continue_final):
            ids.append(EOT)
    if add_generation_prompt and not continue_final:
        ids += CHAT_HEADER
    return ids


def reference(prompt, max_tokens: int):
    """Uninterrupted greedy completion: (ids, text)."""
    seq = tokenize(prompt) if isinstance(prompt, str) else list(prompt)
    out = []
    for _ in range(max_tokens):
        seq.append(next_token(seq))
        out.append(seq[-1])
    return out, "".join(detok(t) for t in out)


class FakeBackend:
    def __init__(self, tpot_ms: float = 0.0, ttft_ms: float = 0.0, model: str = "fake", stamp: bool = False):
        self.tpot = tpot_ms / 1000
        self.ttft = ttft_ms / 1000
        self.model = model
        self.stamp = stamp
        self.fail = None
        self.fail_count = None
        self.requests = []
        self.runner = None
        self.port = None
        self.url = None

    def _take_fail(self):
        if self.fail is None:
            return None
        if self.fail_count is not None:
            if self.fail_count <= 0:
                return None
            self.fail_count -= 1
        return self.fail

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
        p = b["prompt"]
        return await self._generate(req, b, list(p) if isinstance(p, list) else tokenize(p), chat=False)

    async def _chat(self, req):
        b = await req.json()
        self.requests.append(b)
        ids = chat_ids(b["messages"], b.get("add_generation_prompt", True), b.get("continue_final_message", False))
        return await self._generate(req, b, ids, chat=True)

    async def _generate(self, req, b, ids, chat: bool):
        fail = self._take_fail()
        if fail and fail[0] == "http500":
            return web.json_response({"error": "injected failure"}, status=500)
        if b.get("max_tokens") is not None and b["max_tokens"] <= 0:
            return web.json_response({"error": "max_tokens must be positive"}, status=400)
        n_max = b.get("max_tokens") or b.get("max_completion_tokens") or 16
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{len(self.requests)}"
        created = int(time.time())
        want_lp = b.get("logprobs") is not None and b.get("logprobs") is not False
        as_ids = bool(b.get("return_tokens_as_token_ids"))
        want_ids = bool(b.get("return_token_ids"))
        so = b.get("stream_options") or {}
        seq, gen = list(ids), []
        for _ in range(n_max):
            seq.append(next_token(seq))
            gen.append(seq[-1])
        kind = "chat.completion.chunk" if chat else "text_completion"

        def usage(k):
            return {"prompt_tokens": len(ids), "completion_tokens": k, "total_tokens": len(ids) + k}

        def lp(t):
            tok = f"token_id:{t}" if as_ids else detok(t)
            if chat:
                return {"content": [{"token": tok, "logprob": -0.25, "top_logprobs": []}]}
            return {"tokens": [tok], "token_logprobs": [-0.25], "top_logprobs": None, "text_offset": [0]}

        if not b.get("stream"):
            text = "".join(detok(t) for t in gen)
            choice = ({"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": "length"}
                      if chat else {"index": 0, "text": text, "finish_reason": "length", "logprobs": None})
            return web.json_response({"id": rid, "object": "chat.completion" if chat else "text_completion",
                                      "created": created, "model": self.model, "choices": [choice],
                                      "usage": usage(len(gen))})
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream"})
        await resp.prepare(req)

        async def send(obj):
            await resp.write(b"data: " + json.dumps(obj).encode() + b"\n\n")

        if self.ttft:
            await asyncio.sleep(self.ttft)
        if fail and fail[0] == "stall" and fail[1] == 0:
            await asyncio.sleep(3600)
        if chat:
            head = {"id": rid, "object": kind, "created": created, "model": self.model,
                    "choices": [{"index": 0, "delta": {"role": "assistant", "content": ""}, "logprobs": None,
                                 "finish_reason": None}]}
            if so.get("continuous_usage_stats"):
                head["usage"] = usage(0)
            await send(head)
        for k, t in enumerate(gen):
            if fail and fail[1] == k:
                if fail[0] == "reset":
                    await asyncio.sleep(0.02)       # let the chunks already written leave
                    req.transport.abort()
                    return resp
                if fail[0] == "stall":
                    await asyncio.sleep(3600)
            fin = "length" if k == len(gen) - 1 else None
            if chat:
                ch = {"index": 0, "delta": {"content": detok(t)}, "logprobs": lp(t) if want_lp else None,
                      "finish_reason": fin}
            else:
                ch = {"index": 0, "text": detok(t), "logprobs": lp(t) if want_lp else None, "finish_reason": fin,
                      "stop_reason": None}
            if want_ids:
                ch["token_ids"] = [t]
            obj = {"id": rid, "object": kind, "created": created, "model": self.model, "choices": [ch]}
            if so.get("continuous_usage_stats"):
                obj["usage"] = usage(k + 1)
            if self.stamp:
                obj["_t"] = time.time()
            await send(obj)
            if self.tpot:
                await asyncio.sleep(self.tpot)
        if so.get("include_usage"):
            await send({"id": rid, "object": kind, "created": created, "model": self.model, "choices": [],
                        "usage": usage(len(gen))})
        await resp.write(b"data: [DONE]\n\n")
        return resp


class FakePDBackend(FakeBackend):
    """Fake prefill (``role="prefill"``) or decode instance.  Instances of one
    deployment share ``kv`` (transfer id -> held prompt ids + owner) in place of
    the KV connector: a prefill with ``do_remote_decode`` holds its prompt and
    returns ``kv_transfer_params``; a decode with ``do_remote_prefill`` pulls
    the hold and answers 500 if it is gone, its owner is down, or the held ids
    are not the prompt's prefix (wrong KV)."""

    def __init__(self, role: str, kv: dict, **kw):
        super().__init__(**kw)
        self.role = role
        self.kv = kv
        self.alive = True
        self.prefills = 0
        self.pulls = 0

    async def start(self, port=0, host="127.0.0.1"):
        url = await super().start(port, host)
        self.alive = True
        return url

    async def stop(self):
        self.alive = False
        await super().stop()

    async def _generate(self, req, b, ids, chat):
        p = b.get("kv_transfer_params") or {}
        if self.role == "prefill" and p.get("do_remote_decode"):
            fail = self._take_fail()
            if fail and fail[0] == "http500":
                return web.json_response({"error": "injected failure"}, status=500)
            if fail and fail[0] in ("reset", "stall"):
                if fail[0] == "stall":
                    await asyncio.sleep(3600)
                req.transport.abort()
                return web.Response()
            self.prefills += 1
            self.kv[p["transfer_id"]] = {"ids": list(ids), "owner": self}
            return web.json_response({
                "id": "cmpl-prefill", "object": "text_completion", "created": int(time.time()), "model": self.model,
                "choices": [{"index": 0, "text": detok(next_token(ids)), "finish_reason": "length"}],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": 1, "total_tokens": len(ids) + 1},
                "kv_transfer_params": {"do_remote_prefill": True, "do_remote_decode": False,
                                       "transfer_id": p["transfer_id"], "remote_ctrl": self.url,
                                       "remote_num_tokens": len(ids)}})
        if self.role == "decode":
            if not p.get("do_remote_prefill"):
                return web.json_response({"error": "decode instance needs kv_transfer_params"}, status=400)
            held = self.kv.get(p.get("transfer_id"))
            n = p.get("remote_num_tokens", 0)
            if held is None or not held["owner"].alive or len(held["ids"]) != n or held["ids"] != ids[:n]:
                return web.json_response({"error": "KV load failed"}, status=500)
            self.pulls += 1
        return await super()._generate(req, b, ids, chat)


class FakeSGLangPDBackend(FakeBackend):
    """Fake SGLang PD instance: prefill and decode get the request together
    with a ``bootstrap_room``; the decode waits (``wait_s``) for the prefill to
    publish the room in the shared ``rooms`` and fails if it does not or if
    the prefill is down."""

    def __init__(self, role: str, rooms: dict, wait_s: float = 2.0, **kw):
        super().__init__(**kw)
        self.role, self.rooms, self.wait_s = role, rooms, wait_s
        self.alive = True
        self.prefills = 0

    async def start(self, port=0, host="127.0.0.1"):
        url = await super().start(port, host)
        self.alive = True
        return url

    async def stop(self):
        self.alive = False
        await super().stop()

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
        t0 = time.monotonic()
        while room not in self.rooms:
            if time.monotonic() - t0 > self.wait_s:
                return web.json_response({"error": "KV transfer timed out"}, status=500)
            await asyncio.sleep(0.005)
        held, owner = self.rooms[room]
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

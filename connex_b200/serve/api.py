"""OpenAI-compatible HTTP front of a :class:`GenerationEngine` (aiohttp).

Routes: ``/v1/completions`` and ``/v1/chat/completions`` (streamed or
not; ``stream_options.include_usage`` / ``continuous_usage_stats``;
``return_token_ids``; ``return_tokens_as_token_ids``; id prompts; chat
``add_generation_prompt`` / ``continue_final_message``; ``stop`` strings
(held back while they may still match, never shown); ``stop_token_ids``;
``ignore_eos``), ``/tokenize``, ``/detokenize``, ``/v1/models``, ``/health``
(503 once the engine thread has died), ``/load`` (queue and KV reservation
figures) and ``/metrics`` (Prometheus: requests by finish reason, tokens,
TTFT / TPOT histograms, queue and KV gauges).  This is the request surface the retry / resume proxy
and the PD router drive, so both can front this engine directly.

Decoding is greedy (the device argmax); ``temperature`` and friends are
accepted and ignored, ``n`` / ``best_of`` above 1 are refused.  Log
probabilities are not computed: when asked for, each token is listed with
``logprob: null``.

Text codec: an HF tokenizer directory (``tokenizer=``) when given, else the
word codec of the CPU test backend (word ``t<i>`` is id ``i``; text of id
``i`` is ``" t<i>"``), which round-trips every id exactly and needs no files.
"""
from __future__ import annotations

import asyncio
import json
import time
from typing import List

from aiohttp import web

from connex_b200.serve.engine import EngineFull, GenerationEngine

BOS, EOT = 1, 4
CHAT_HEADER = [2, 3]


class WordCodec:
    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size
        self.eos_id = None

    def encode(self, text: str, add_special: bool = True) -> List[int]:
        ids = [BOS] if add_special else []
        for w in text.split():
            if w.startswith("t") and w[1:].isdigit():
                ids.append(int(w[1:]) % self.vocab_size)
            else:
                ids.append(sum(w.encode()) % self.vocab_size)
        return ids

    def decode_one(self, t: int) -> str:
        return f" t{t}"

    def decode(self, ids) -> str:
        return "".join(self.decode_one(int(t)) for t in ids)

    def stream(self) -> "_WordStream":
        return _WordStream(self)

    def chat(self, messages, add_generation_prompt=True, continue_final=False) -> List[int]:
        ids = [BOS]
        for i, m in enumerate(messages):
            ids += CHAT_HEADER + self.encode(m.get("content") or "", add_special=False)
            if not (i == len(messages) - 1 and continue_final):
                ids.append(EOT)
        if add_generation_prompt and not continue_final:
            ids += CHAT_HEADER
        return ids


class HFCodec:
    """A local HF tokenizer (``AutoTokenizer.from_pretrained(path)``, no network)."""

    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_id = self.tok.eos_token_id

    def encode(self, text: str, add_special: bool = True) -> List[int]:
        return list(self.tok.encode(text, add_special_tokens=add_special))

    def decode_one(self, t: int) -> str:
        return self.tok.decode([t], skip_special_tokens=True)

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def stream(self) -> "IncrementalDetokenizer":
        return IncrementalDetokenizer(self.tok)

    def chat(self, messages, add_generation_prompt=True, continue_final=False) -> List[int]:
        out = self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                           continue_final_message=continue_final, tokenize=True)
        if hasattr(out, "keys"):          # newer transformers return a BatchEncoding
            out = out["input_ids"]
        return [int(t) for t in out]


class _WordStream:
    """Per-request text of the word codec: every id is a whole word."""

    def __init__(self, codec: WordCodec):
        self.codec = codec

    def feed(self, t: int) -> str:
        return self.codec.decode_one(t)

    def flush(self) -> str:
        return ""


class IncrementalDetokenizer:
    """Streaming text of one request's generated ids for a subword tokenizer.

    Decoding each id on its own breaks two things: a byte-level BPE splits a
    multi-byte UTF-8 character across ids (each piece alone decodes to
    U+FFFD), and word-initial spaces depend on the previous piece.  So each
    ``feed`` decodes a short window -- the ids already shown since the last
    stable point plus the new ones -- and emits only the text beyond what
    the window's shown part decodes to.  While the window's text ends in an
    incomplete character (U+FFFD) nothing is emitted; the bytes come out
    with the id that completes them.  Special tokens (EOS and the like) are
    skipped."""

    def __init__(self, tok):
        self.tok = tok
        self.ids: List[int] = []
        self.start = 0        # first id of the decoding window (left context)
        self.shown = 0        # ids [start, shown) are already emitted as text

    def _text(self, a: int, b: int) -> str:
        return self.tok.decode(self.ids[a:b], skip_special_tokens=True)

    def feed(self, t: int) -> str:
        self.ids.append(int(t))
        before = self._text(self.start, self.shown)
        now = self._text(self.start, len(self.ids))
        if now.endswith("\ufffd") or len(now) < len(before) or not now.startswith(before):
            return ""                                  # an incomplete character: wait for its next byte
        new = now[len(before):]
        # the ids just shown become the next window's left context
        self.start, self.shown = self.shown, len(self.ids)
        return new

    def flush(self) -> str:
        """Whatever is still held back (an unfinished character at the end)."""
        if self.shown == len(self.ids):
            return ""
        before = self._text(self.start, self.shown)
        now = self._text(self.start, len(self.ids))
        self.shown = len(self.ids)
        return now[len(before):] if now.startswith(before) else now


class StopMatcher:
    """Text stop sequences (the API's ``stop``): ``feed`` returns the text
    that may be shown now and whether a stop sequence completed.  Text that
    could still be the start of a stop sequence is held back until it is not
    (or until ``flush``); the stop sequence itself is never shown."""

    def __init__(self, stops):
        if isinstance(stops, str):
            stops = [stops]
        self.stops = [x for x in (stops or []) if x]
        self.held = ""

    def feed(self, text: str):
        if not self.stops:
            return text, False
        buf = self.held + text
        hits = [(buf.find(x), x) for x in self.stops if x in buf]
        if hits:
            at = min(i for i, _ in hits)
            self.held = ""
            return buf[:at], True
        keep = 0
        for x in self.stops:
            for n in range(min(len(x) - 1, len(buf)), 0, -1):
                if buf.endswith(x[:n]):
                    keep = max(keep, n)
                    break
        self.held = buf[len(buf) - keep:] if keep else ""
        return buf[:len(buf) - keep], False

    def flush(self) -> str:
        out, self.held = self.held, ""
        return out


def _err(msg: str, status: int = 400) -> web.Response:
    return web.json_response({"error": {"message": msg, "type": "invalid_request_error", "code": status}},
                             status=status)


class _Metrics:
    """Prometheus collectors of one server (own registry, so several servers
    can live in one process): requests by outcome, generated tokens, TTFT
    and TPOT histograms, and the engine's queue / KV gauges read at scrape."""

    def __init__(self, engine: GenerationEngine):
        from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram
        self.registry = r = CollectorRegistry()
        self.requests = Counter("connex_serve_requests", "finished requests", ["finish_reason"], registry=r)
        self.tokens = Counter("connex_serve_generated_tokens", "generated tokens", registry=r)
        self.ttft = Histogram("connex_serve_ttft_seconds", "arrival to first token", registry=r,
                              buckets=(.005, .01, .025, .05, .1, .25, .5, 1, 2.5, 5, 10))
        self.tpot = Histogram("connex_serve_tpot_seconds", "mean time per output token after the first",
                              registry=r, buckets=(.001, .0025, .005, .01, .02, .05, .1, .25))
        for name, key in (("waiting", "waiting"), ("running", "running"), ("kv_blocks_reserved", "kv_blocks_reserved"),
                          ("kv_blocks", "kv_blocks")):
            g = Gauge(f"connex_serve_{name}", name.replace("_", " "), registry=r)
            g.set_function(lambda key=key: engine.load()[key])

    def finished(self, req, reason: str) -> None:
        self.requests.labels(reason or "unknown").inc()
        self.tokens.inc(len(req.gen))
        if req.t_first is not None:
            self.ttft.observe(req.t_first - req.t_submit)
            if len(req.gen) > 1:
                import time as _t
                self.tpot.observe((_t.monotonic() - req.t_first) / (len(req.gen) - 1))


class Server:
    def __init__(self, engine: GenerationEngine, model: str = "connex-b200", codec=None):
        self.engine = engine
        self.model = model
        self.codec = codec or WordCodec(engine.s.vocab_size or 1000)
        self._n = 0
        try:
            self.metrics = _Metrics(engine)
        except ImportError:          # prometheus_client is optional
            self.metrics = None

    def app(self) -> web.Application:
        app = web.Application(client_max_size=64 << 20)
        app.router.add_post("/v1/completions", self._completions)
        app.router.add_post("/v1/chat/completions", self._chat)
        app.router.add_post("/tokenize", self._tokenize)
        app.router.add_post("/detokenize", self._detokenize)
        app.router.add_get("/v1/models", self._models)
        app.router.add_get("/health", self._health)
        app.router.add_get("/load", self._load)
        app.router.add_get("/metrics", self._metrics)
        return app

    async def _metrics(self, req):
        if self.metrics is None:
            return web.Response(status=404, text="prometheus_client is not installed")
        from prometheus_client import CONTENT_TYPE_LATEST, generate_latest
        return web.Response(body=generate_latest(self.metrics.registry),
                            headers={"Content-Type": CONTENT_TYPE_LATEST})

    async def _models(self, req):
        return web.json_response({"object": "list", "data": [{"id": self.model, "object": "model",
                                                              "max_model_len": self.engine.s.max_ctx}]})

    async def _health(self, req):
        if not self.engine.alive:
            return web.json_response({"status": "engine down", "error": self.engine.error}, status=503)
        return web.json_response({"status": "ok"})

    async def _load(self, req):
        return web.json_response({**self.engine.load(), **{k: v for k, v in self.engine.stats.items()}})

    async def _tokenize(self, req):
        b = await req.json()
        if "messages" in b:
            ids = self.codec.chat(b["messages"], b.get("add_generation_prompt", True),
                                  b.get("continue_final_message", False))
        else:
            ids = self.codec.encode(b["prompt"], b.get("add_special_tokens", True))
        return web.json_response({"tokens": ids, "count": len(ids), "max_model_len": self.engine.s.max_ctx})

    async def _detokenize(self, req):
        b = await req.json()
        return web.json_response({"prompt": self.codec.decode([int(t) for t in b["tokens"]])})

    async def _completions(self, req):
        try:
            b = await req.json()
        except json.JSONDecodeError:
            return _err("body is not JSON")
        p = b.get("prompt")
        if isinstance(p, list) and len(p) == 1 and isinstance(p[0], (str, list)):
            p = p[0]
        if isinstance(p, str):
            ids = self.codec.encode(p)
        elif isinstance(p, list) and p and all(isinstance(t, int) for t in p):
            ids = list(p)
        else:
            return _err("prompt must be a string or a list of token ids (one prompt per request)")
        return await self._generate(req, b, ids, chat=False)

    async def _chat(self, req):
        try:
            b = await req.json()
        except json.JSONDecodeError:
            return _err("body is not JSON")
        if not isinstance(b.get("messages"), list) or not b["messages"]:
            return _err("messages must be a non-empty list")
        ids = self.codec.chat(b["messages"], b.get("add_generation_prompt", True), b.get("continue_final_message",
                                                                                         False))
        return await self._generate(req, b, ids, chat=True)

    async def _generate(self, req, b, ids, chat: bool):
        if (b.get("n") or 1) != 1 or (b.get("best_of") or 1) != 1:
            return _err("n / best_of above 1 are not supported (greedy decoding)")
        n_max = b.get("max_tokens") if b.get("max_tokens") is not None else b.get("max_completion_tokens")
        n_max = 16 if n_max is None else int(n_max)
        stop = set(int(t) for t in (b.get("stop_token_ids") or []))
        if self.codec.eos_id is not None and not b.get("ignore_eos"):
            stop.add(int(self.codec.eos_id))
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        metrics = self.metrics

        def on_token(r, tok, reason):
            if reason is not None and metrics is not None:
                metrics.finished(r, reason)
            loop.call_soon_threadsafe(q.put_nowait, (tok, reason))
        try:
            r = self.engine.submit(ids, n_max, on_token, stop_ids=stop)
        except (ValueError, EngineFull) as e:
            return _err(str(e))
        self._n += 1
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{self._n}-{r.rid}"
        created = int(time.time())
        want_lp = b.get("logprobs") is not None and b.get("logprobs") is not False
        as_ids = bool(b.get("return_tokens_as_token_ids"))
        want_ids = bool(b.get("return_token_ids"))
        so = b.get("stream_options") or {}
        kind = "chat.completion.chunk" if chat else "text_completion"

        def usage(k):
            return {"prompt_tokens": len(ids), "completion_tokens": k, "total_tokens": len(ids) + k}

        def lp(t):
            tok = f"token_id:{t}" if as_ids else self.codec.decode_one(t)
            if chat:
                return {"content": [{"token": tok, "logprob": None, "top_logprobs": []}]}
            return {"tokens": [tok], "token_logprobs": [None], "top_logprobs": None, "text_offset": [0]}

        sm = StopMatcher(b.get("stop"))
        dt = self.codec.stream()

        def text_of(tok, reason):
            """New text of a generated id; a stop id ends the output without text."""
            if reason == "stop" and tok in stop:
                return dt.flush()
            return dt.feed(tok) + (dt.flush() if reason is not None else "")
        if not b.get("stream"):
            toks, reason, parts = [], None, []
            try:
                while reason is None:
                    tok, reason = await q.get()
                    if tok is not None:
                        toks.append(tok)
                        shown, hit = sm.feed(text_of(tok, reason))
                        parts.append(shown)
                        if hit:
                            self.engine.cancel(r)
                            reason = "stop"
            except asyncio.CancelledError:
                self.engine.cancel(r)
                raise
            if reason in ("error", "abort"):
                return _err(f"generation failed: {r.error or reason}", 500)
            text = "".join(parts) + sm.flush()
            if chat:
                choice = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": reason}
            else:
                choice = {"index": 0, "text": text, "finish_reason": reason, "logprobs": None}
            if want_ids:
                choice["token_ids"] = toks
            return web.json_response({"id": rid, "object": "chat.completion" if chat else "text_completion",
                                      "created": created, "model": self.model, "choices": [choice],
                                      "usage": usage(len(toks))})
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
        await resp.prepare(req)

        async def send(obj):
            await resp.write(b"data: " + json.dumps(obj).encode() + b"\n\n")
        k = 0
        try:
            if chat:
                head = {"id": rid, "object": kind, "created": created, "model": self.model,
                        "choices": [{"index": 0, "delta": {"role": "assistant", "content": ""}, "logprobs": None,
                                     "finish_reason": None}]}
                if so.get("continuous_usage_stats"):
                    head["usage"] = usage(0)
                await send(head)
            reason = None
            while reason is None:
                tok, reason = await q.get()
                if tok is None:
                    # ended without a token: tell the client and drop the stream without [DONE]
                    await send({"id": rid, "object": kind, "created": created, "model": self.model,
                                "choices": [], "error": {"message": r.error or reason}})
                    if req.transport is not None:
                        req.transport.abort()
                    return resp
                k += 1
                shown, hit = sm.feed(text_of(tok, reason))
                if hit:
                    self.engine.cancel(r)
                    reason = "stop"
                elif reason is not None:
                    shown += sm.flush()
                if chat:
                    ch = {"index": 0, "delta": {"content": shown},
                          "logprobs": lp(tok) if want_lp else None, "finish_reason": reason}
                else:
                    ch = {"index": 0, "text": shown, "logprobs": lp(tok) if want_lp else None,
                          "finish_reason": reason, "stop_reason": None}
                if want_ids:
                    ch["token_ids"] = [tok]
                obj = {"id": rid, "object": kind, "created": created, "model": self.model, "choices": [ch]}
                if so.get("continuous_usage_stats"):
                    obj["usage"] = usage(k)
                await send(obj)
            if so.get("include_usage"):
                await send({"id": rid, "object": kind, "created": created, "model": self.model, "choices": [],
                            "usage": usage(k)})
            await resp.write(b"data: [DONE]\n\n")
        except (ConnectionResetError, asyncio.CancelledError):
            self.engine.cancel(r)
            raise
        return resp


async def serve(server: Server, host: str = "0.0.0.0", port: int = 8100):
    """Start the HTTP server; returns (runner, bound port)."""
    runner = web.AppRunner(server.app(), shutdown_timeout=1.0)
    await runner.setup()
    site = web.TCPSite(runner, host, port)
    await site.start()
    return runner, site._server.sockets[0].getsockname()[1]

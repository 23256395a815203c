"""Closed-loop serving benchmark through the OpenAI API of this framework's
engine (``connex_b200.serve``): C clients each stream completions back to
back (random token-id prompts of ``--prompt-len``, ``--max-tokens`` greedy
output tokens) for ``--duration-s``; reported per concurrency: output
tokens/s, requests/s, TTFT and TPOT percentiles (client-side wall clock,
the way a user sees them; the server runs in this process on one GPU).

    python -m connex_b200.bench.serve_bench --clients 1,32 --prompt-len 1024 --max-tokens 128

Reference counterparts: the PP closed-loop and upstream-vLLM PP=2 C=1 / C=32
tok/s and TPOT rows of ``docs/results.md`` (there on A40s through vLLM).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import time


def _pct(xs, q):
    if not xs:
        return None
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(q * len(xs)))]


async def _client(url, prompt_len, max_tokens, vocab, deadline, rng, out, min_requests=0):
    import aiohttp
    mine = 0
    async with aiohttp.ClientSession() as s:
        while time.monotonic() < deadline or mine < min_requests:
            mine += 1
            prompt = [rng.randrange(16, vocab) for _ in range(prompt_len)]
            t0 = time.monotonic()
            first, n, stamps = None, 0, []
            async with s.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": max_tokens,
                                                             "stream": True, "ignore_eos": True}) as r:
                if r.status != 200:
                    out["errors"] += 1
                    continue
                async for line in r.content:
                    line = line.strip()
                    if not line.startswith(b"data:") or line[5:].strip() == b"[DONE]":
                        continue
                    now = time.monotonic()
                    if first is None:
                        first = now
                    stamps.append(now)
                    n += 1
            if n == 0:
                out["errors"] += 1
                continue
            out["ttft"].append(first - t0)
            if n > 1:
                out["tpot"].append((stamps[-1] - first) / (n - 1))
            out["tokens"] += n
            out["requests"] += 1
            out["done_t"].append(time.monotonic())


async def run_level(url, clients, prompt_len, max_tokens, vocab, duration_s, seed=0, min_requests=0):
    out = {"ttft": [], "tpot": [], "tokens": 0, "requests": 0, "errors": 0, "done_t": []}
    t0 = time.monotonic()
    deadline = t0 + duration_s
    await asyncio.gather(*[_client(url, prompt_len, max_tokens, vocab, deadline, random.Random(seed * 1000 + c), out,
                                   min_requests) for c in range(clients)])
    wall = time.monotonic() - t0
    return {"clients": clients, "requests": out["requests"], "errors": out["errors"], "wall_s": round(wall, 2),
            "output_tok_s": round(out["tokens"] / wall, 1), "req_s": round(out["requests"] / wall, 3),
            "ttft_p50_ms": round(1e3 * _pct(out["ttft"], 0.5), 1) if out["ttft"] else None,
            "ttft_p99_ms": round(1e3 * _pct(out["ttft"], 0.99), 1) if out["ttft"] else None,
            "tpot_p50_ms": round(1e3 * _pct(out["tpot"], 0.5), 2) if out["tpot"] else None,
            "tpot_mean_ms": round(1e3 * statistics.mean(out["tpot"]), 2) if out["tpot"] else None}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", default="llama3-8b", choices=["llama3-8b", "llama3.1-8b", "tiny"])
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--clients", default="1,32")
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--duration-s", type=float, default=20.0)
    ap.add_argument("--warmup-requests", type=int, default=3)
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--num-blocks", type=int, default=0)
    ap.add_argument("--rule", action="store_true", help="CPU stand-in model (wiring check)")
    ap.add_argument("--no-graphs", action="store_true", help="eager decode steps (no CUDA graphs)")
    a = ap.parse_args(argv)
    from connex_b200.serve.__main__ import build_stepper
    from connex_b200.serve.api import Server, serve
    from connex_b200.serve.engine import GenerationEngine
    ns = argparse.Namespace(rule=a.rule, checkpoint=a.checkpoint, config=a.config, layers=None, seed=0,
                            device="cuda:0", num_blocks=a.num_blocks, kv_fraction=0.8, max_batch=a.max_batch,
                            max_ctx=a.prompt_len + a.max_tokens + 64, max_step_tokens=max(8192, a.prompt_len + 64),
                            num_stages=1, stage_starts=None, directory=None, data="link", store=None,
                            store_master=False, replica=0, advertise_host="127.0.0.1", recv_timeout_s=30.0,
                            no_graphs=a.no_graphs, tp=1)
    stepper, _ = build_stepper(ns)
    engine = GenerationEngine(stepper).start()
    server = Server(engine, "bench")
    vocab = stepper.vocab_size or 1000
    results = []

    async def go():
        runner, port = await serve(server, "127.0.0.1", 0)
        url = f"http://127.0.0.1:{port}"
        try:
            await run_level(url, 1, a.prompt_len, 8, vocab, 0.0, min_requests=a.warmup_requests)   # first touch
            for c in [int(x) for x in a.clients.split(",")]:
                r = await run_level(url, c, a.prompt_len, a.max_tokens, vocab, a.duration_s, seed=c)
                r.update(engine_prefill_steps=engine.stats["prefill_steps"],
                         engine_decode_steps=engine.stats["decode_steps"])
                results.append(r)
                print(json.dumps({"serve_bench": r}), flush=True)
        finally:
            await runner.cleanup()
    try:
        asyncio.run(go())
    finally:
        engine.stop()
    print(json.dumps({"metric": "serving output tok/s (closed loop, OpenAI API, 1 GPU)",
                      "model": a.checkpoint or a.config, "prompt_len": a.prompt_len, "max_tokens": a.max_tokens,
                      "levels": results}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

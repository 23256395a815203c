"""Added latency of the retry / resume proxy (``connex-proxy``) on CPU: a
fake OpenAI backend whose chunks carry their send time (``--stamp``) and the
proxy run as separate processes; the same closed-loop load (``--concurrency``
streams of ``--tokens`` tokens, ``--tpot-ms`` apart) is sent straight to the
backend and through the proxy, alternating passes.  Per chunk: client
receive time - backend send time; the report gives p50 / p99 for both paths
(and p99 without each stream's first 4 chunks, the arrival burst), the
proxy's added p50, and mean end-to-end request time for both.

    python -m connex_b200.bench.proxy_overhead --requests 200 --concurrency 16 --tokens 64 --tpot-ms 10

Reference counterpart: ``benchmarks/proxy_overhead.py``.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import socket
import subprocess
import sys
import time


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pct(xs, q):
    xs = sorted(xs)
    return round(xs[min(len(xs) - 1, int(q * len(xs)))] * 1e3, 3) if xs else None


async def _up(url: str, timeout_s: float = 30.0) -> None:
    import aiohttp
    end = time.monotonic() + timeout_s
    async with aiohttp.ClientSession() as s:
        while True:
            try:
                async with s.get(url + "/v1/models") as r:
                    if r.status == 200:
                        return
            except aiohttp.ClientError:
                pass
            if time.monotonic() > end:
                raise TimeoutError(url)
            await asyncio.sleep(0.1)


async def _load(url: str, n: int, conc: int, tokens: int) -> dict:
    import aiohttp
    chunk_lat, steady, e2e = [], [], []
    sem = asyncio.Semaphore(conc)

    async def one(s, k):
        async with sem:
            t0 = time.time()
            idx = 0
            async with s.post(url + "/v1/completions", json={"model": "fake", "prompt": f"t{k} t{k + 1}",
                                                             "max_tokens": tokens, "stream": True}) as r:
                async for line in r.content:
                    line = line.strip()
                    if not line.startswith(b"data:") or line[5:].strip() == b"[DONE]":
                        continue
                    c = json.loads(line[5:])
                    if "_t" in c:
                        d = time.time() - c["_t"]
                        chunk_lat.append(d)
                        if idx >= 4:
                            steady.append(d)
                        idx += 1
            e2e.append(time.time() - t0)
    async with aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=conc * 2)) as s:
        await asyncio.gather(*[one(s, k) for k in range(n)])
    return {"p50_ms": _pct(chunk_lat, 0.5), "p99_ms": _pct(chunk_lat, 0.99), "steady_p99_ms": _pct(steady, 0.99),
            "e2e_mean_s": round(sum(e2e) / len(e2e), 4), "chunks": len(chunk_lat)}


def bench(requests: int, concurrency: int, tokens: int, tpot_ms: float, passes: int = 2) -> dict:
    bp, pp = _port(), _port()
    backend = subprocess.Popen([sys.executable, "-m", "connex.serving.fake_backend", "--port", str(bp), "--tpot-ms",
                                str(tpot_ms), "--stamp"], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    proxy = subprocess.Popen([sys.executable, "-m", "connex.serving.proxy", "--host", "127.0.0.1", "--port", str(pp),
                              "--endpoints", f"http://127.0.0.1:{bp}", "--log-level", "WARNING"],
                             stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    direct_url, proxy_url = f"http://127.0.0.1:{bp}", f"http://127.0.0.1:{pp}"
    try:
        async def go():
            await _up(direct_url)
            await _up(proxy_url)
            res = {"direct": [], "proxy": []}
            for _ in range(passes):
                res["direct"].append(await _load(direct_url, requests, concurrency, tokens))
                res["proxy"].append(await _load(proxy_url, requests, concurrency, tokens))
            return res
        res = asyncio.run(go())
    finally:
        for p in (proxy, backend):
            p.terminate()
            p.wait(10)
    d, p = res["direct"][-1], res["proxy"][-1]
    return {"requests": requests, "concurrency": concurrency, "tokens": tokens, "tpot_ms": tpot_ms,
            "direct": d, "proxy": p, "added_p50_ms": round(p["p50_ms"] - d["p50_ms"], 3),
            "added_e2e_mean_s": round(p["e2e_mean_s"] - d["e2e_mean_s"], 4)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--requests", type=int, default=200)
    ap.add_argument("--concurrency", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--tpot-ms", type=float, default=10.0)
    ap.add_argument("--passes", type=int, default=2)
    a = ap.parse_args(argv)
    print(json.dumps(bench(a.requests, a.concurrency, a.tokens, a.tpot_ms, a.passes)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

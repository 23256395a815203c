"""Reference arm of the flagship benchmark: the unmodified reference's PD KV
hand-off, run through its own public API on this machine.

Run by ``bench.py --impl reference`` in an isolated interpreter whose import
path holds only the installed reference (``baseline/_ref``): nothing of this
repository is imported here.  The reference moves a request's paged KV with
``connex.pd.transfer.KVProducer.hold`` on the prefill side and
``KVConsumer.pull`` on the decode side.  Its GPU data planes are connex-rs
(an external Rust/UCX engine) and Mooncake; neither is installed, and the
machine has no GPUDirect peer-memory driver, so the reference's stock
selection stages the KV through pinned host memory (``host_staging``:
device -> host mirror on the prefill GPU, host copy between the mirrors by
its in-process ``loopback`` plane, host mirror -> device on the decode GPU).
That is the path measured.

Workload (the flagship's): Llama-3-8B KV geometry (32 layers x 8 KV heads x
128, bf16, 16-token blocks, one ``[2, blocks, 8, 16, 128]`` tensor per layer
as vLLM lays it out), per step ``--batch`` prompts whose lengths are drawn
exactly as the flagship draws them (uniform 512-8192, seed 0), random KV
contents.  There is no model in the reference, so there is no prefill
compute; a step is the hand-off of the step's prompts' KV.

Per step (host clock, both GPUs synchronized on both sides):
* ``pull_s``  -- the consumer's own pull time (acquire, meta, the plane's
  copy, the copy back to the device) of the step's concurrent pulls (the
  longest); summed bytes / summed seconds = ``value``;
* ``step_s``  -- hold (including the device -> host staging) until every
  pull is done = ``e2e``.

Prints one JSON object per rank; ``bench.py`` aggregates.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--ref", required=True, help="directory of the installed reference")
    p.add_argument("--src-device", type=int, default=0)
    p.add_argument("--dst-device", type=int, default=0)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--min-len", type=int, default=512)
    p.add_argument("--max-len", type=int, default=8192)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args()
    sys.path.insert(0, a.ref)
    os.environ.setdefault("CONNEX_PD_BACKEND", "loopback")

    import numpy as np
    import torch
    from connex.pd.dataplane import make_plane
    from connex.pd.kv_layout import tensor_layout
    from connex.pd.transfer import KVConsumer, KVProducer
    import connex
    assert os.path.abspath(a.ref) in os.path.abspath(connex.__file__), "not the installed reference"

    L, H, BS, D = a.layers, 8, 16, 128
    per_seq = (a.max_len + BS) // BS + 1
    n_blocks = a.batch * per_seq + 16
    sdev, ddev = torch.device("cuda", a.src_device), torch.device("cuda", a.dst_device)

    def cache(dev):
        g = torch.Generator(device=dev)
        g.manual_seed(1234 + dev.index)
        return [torch.randn(2, n_blocks, H, BS, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(L)]

    with torch.cuda.device(sdev):
        src = cache(sdev)
        producer = KVProducer(make_plane("bench", 0, 0, 0, "127.0.0.1", backend="loopback"),
                              [tensor_layout(t, n_blocks) for t in src], bind_ip="127.0.0.1", block_size=BS)
    with torch.cuda.device(ddev):
        dst = [torch.zeros_like(t, device=ddev) for t in src]
        consumer = KVConsumer(make_plane("bench", 1, 0, 0, "127.0.0.1", backend="loopback"),
                              [tensor_layout(t, n_blocks) for t in dst], block_size=BS)
    addr = f"127.0.0.1:{producer.port}"
    block_bytes = L * 2 * H * BS * D * 2

    def sync():
        torch.cuda.synchronize(sdev)
        torch.cuda.synchronize(ddev)

    def step(s: int, check: bool = False):
        rng = np.random.default_rng([a.seed, s])
        lens = [int(n) for n in rng.integers(a.min_len, a.max_len + 1, size=a.batch)]
        need = [(n + BS - 1) // BS for n in lens]
        sblocks, dblocks, off = [], [], 0
        for k in need:                       # source blocks in order; destination blocks reversed
            sblocks.append(list(range(off, off + k)))
            dblocks.append(list(range(n_blocks - 1 - off, n_blocks - 1 - off - k, -1)))
            off += k
        sync()
        t0 = time.perf_counter()
        with torch.cuda.device(sdev):
            for i, sb in enumerate(sblocks):
                producer.hold(f"r{s}-{i}", f"t{s}-{i}", sb)
        for i, db in enumerate(dblocks):
            consumer.pull(f"r{s}-{i}", addr, f"t{s}-{i}", db)
        got = []
        while len(got) < len(dblocks):
            got += consumer.take_done()
            time.sleep(0.0002)
        sync()
        step_s = time.perf_counter() - t0
        bad = [r for r in got if not r.ok]
        if bad:
            raise SystemExit(f"reference pull failed: {bad[0].why}")
        ok = True
        if check:
            for sb, db in zip(sblocks, dblocks):
                si = torch.tensor(sb, device=sdev)
                di = torch.tensor(db, device=ddev)
                for l in range(L):
                    if not torch.equal(src[l].index_select(1, si).cpu(), dst[l].index_select(1, di).cpu()):
                        ok = False
        for i in range(len(dblocks)):
            consumer.release(addr, f"t{s}-{i}")
        deadline = time.monotonic() + 10
        while producer.held() and time.monotonic() < deadline:
            producer.take_finished()
            time.sleep(0.001)
        return {"bytes": sum(need) * block_bytes, "pull_s": max(r.seconds for r in got), "step_s": step_s,
                "tokens": sum(lens), "ok": ok}

    for w in range(a.warmup):
        step(10_000 + w)
    recs = [step(s) for s in range(a.steps)]
    chk = step(20_000, check=True)
    consumer.close()
    producer.close()
    print(json.dumps({"recs": recs, "kv_check": chk["ok"], "src": a.src_device, "dst": a.dst_device}), flush=True)


if __name__ == "__main__":
    main()

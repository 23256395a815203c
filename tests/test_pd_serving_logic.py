"""Host protocol of the PD serving benchmark on CPU: the prefill side (decode
block allocator, KV leases, re-push after a decode death) and the decode side
(continuous batching, admission, kill and replacement) run as two threads
over a ZeroMQ pair, with the model, the KV push and the device waits replaced
by stand-ins.  Every request must complete exactly once; after the kill every
lost request is refilled and decodes again."""
import threading
import types

import pytest
import torch
import zmq

from connex_b200.bench import pd_serving_bench as B
from connex_b200.models.llama import LlamaConfig


class FakeModel:
    def __init__(self, *a, **kw):
        pass

    def prefill(self, ids, positions, slots, seq_lens, last_rows, tile_info, layer_hook=None):
        if layer_hook is not None:
            for layer in range(2):
                layer_hook(layer)
        return torch.arange(len(seq_lens), dtype=torch.int32) + 100


class FakePusher:
    def __init__(self, cache, max_ctas=0):
        self.status, self.launched, self.bytes = None, 0, 0

    def begin(self, pairs, dst, timing=False):
        self.launched, self.bytes, self.pairs = 0, 0, pairs

    def hook(self, layer):
        self.launched += 1
        self.bytes += 4096 * len(self.pairs)

    def join(self):
        pass

    def push_ms(self):
        return 0.01


def _batch(cache, prompts, dev, ids=None):
    blocks = [cache.allocate(cache.blocks_needed(len(p))) for p in prompts]
    return types.SimpleNamespace(src_blocks=blocks, seq_lens=[len(p) for p in prompts], ids=None, positions=None,
                                 slots=None, last_rows=None, tile_info=None)


class FakeReady:
    def data_ptr(self):
        return 0


@pytest.fixture
def stubbed(monkeypatch):
    waits = []
    monkeypatch.setattr(B, "LlamaModel", FakeModel)
    monkeypatch.setattr(B, "LayerwiseKVPusher", FakePusher)
    monkeypatch.setattr(B, "build_prefill_batch", _batch)
    monkeypatch.setattr(B, "block_pairs", lambda s, d, dev: [p for a, b in zip(s, d) for p in zip(a, b)])
    monkeypatch.setattr(B, "DecodeBatch", lambda cache, blocks, ctx, dev: types.SimpleNamespace(B=len(blocks)))
    monkeypatch.setattr(B, "decode_step", lambda model, batch, ids, ws: ids + 1)
    monkeypatch.setattr(B.ops, "wait_flag", lambda addr, target, status, timeout_s=0: waits.append(target))
    monkeypatch.setattr(B.ops, "check_status", lambda *a: None)
    monkeypatch.setattr(B.ops, "decode_workspace", lambda *a: None)
    monkeypatch.setattr(B.ops, "new_status", lambda dev: None)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    return waits


def _run(kill_at: float):
    cfg = LlamaConfig.tiny(layers=2)
    args = types.SimpleNamespace(qps=200.0, duration=0.25, min_len=16, max_len=64, out_tokens=8, token_budget=128,
                                 max_running=8, prefill_blocks=64, decode_blocks=64, layers=2, seed=0, pair=0,
                                 kill_at=kill_at, restart_s=0.02)
    ctx = zmq.Context()
    a, b = ctx.socket(zmq.PAIR), ctx.socket(zmq.PAIR)
    a.bind("inproc://serving")
    b.connect("inproc://serving")
    out = {}

    def pre():
        out["pre"] = B.prefill_side(args, cfg, None, torch.device("cpu"), a, None, args.decode_blocks)

    def dec():
        cache = types.SimpleNamespace()
        out["dec"] = B.decode_side(args, cfg, None, torch.device("cpu"), b, cache, FakeReady())
    ts = [threading.Thread(target=pre), threading.Thread(target=dec)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    a.close(0)
    b.close(0)
    ctx.term()
    assert not any(t.is_alive() for t in ts), "the serving protocol did not finish"
    return args, out


def test_every_request_completes_once(stubbed):
    args, out = _run(kill_at=0.0)
    n = out["pre"]["requests"]
    assert n > 10 and out["dec"]["completed"] == n and len(out["dec"]["ttft_ms"]) == n
    assert out["dec"]["output_tokens"] == n * args.out_tokens and out["pre"]["repushed"] == 0
    assert stubbed == sorted(stubbed)                  # cumulative ready targets only grow


def test_decode_death_refills_the_replacement_from_held_kv(stubbed):
    args, out = _run(kill_at=0.12)
    n, lost = out["pre"]["requests"], out["dec"]["lost"]
    assert lost > 0 and out["pre"]["repushed"] == lost and len(out["dec"]["stall_ms"]) == lost
    assert out["dec"]["completed"] == n                 # lost requests complete after the refill
    assert len(out["dec"]["ttft_ms"]) + 0 <= n and min(out["dec"]["stall_ms"]) >= args.restart_s * 1e3

"""Tensor parallelism: the shards recombine into the full weights, the
sharded fp32 computation with exact partial sums equals the unsharded
forward, shapes that do not split are refused, and the row-parallel GEMM's
all-reduce trick (rank 0 adds the residual, the others store partials) gives
x + a @ w^T on every rank of a 2-rank gloo group.  On 2 GPUs the native
kernels with NCCL all-reduces follow the fp32 forward."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from connex_b200 import ops
from connex_b200.models.llama import LlamaConfig, LlamaWeights, reference_forward
from connex_b200.parallel.tp import TPGroup, reference_tp_forward, shard_llama, tp_config
from tests.helpers import free_port

CFG = LlamaConfig.tiny(layers=2)


def test_shards_recombine():
    w = LlamaWeights.random(CFG, "cpu", seed=1, std=0.05)
    sh = [shard_llama(w, r, 2) for r in range(2)]
    c = sh[0].cfg
    assert (c.heads, c.kv_heads, c.ffn) == (CFG.heads // 2, CFG.kv_heads // 2, CFG.ffn // 2)
    for li, lw in enumerate(w.layers):
        q = torch.cat([s.layers[li].wqkv[:c.heads * 128] for s in sh])
        k = torch.cat([s.layers[li].wqkv[c.heads * 128:(c.heads + c.kv_heads) * 128] for s in sh])
        v = torch.cat([s.layers[li].wqkv[(c.heads + c.kv_heads) * 128:] for s in sh])
        assert torch.equal(torch.cat([q, k, v]), lw.wqkv)
        assert torch.equal(torch.cat([s.layers[li].wo for s in sh], 1), lw.wo)
        assert torch.equal(torch.cat([s.layers[li].w2 for s in sh], 1), lw.w2)
        g, u = ops.deinterleave_gate_up(lw.w13)
        parts = [ops.deinterleave_gate_up(s.layers[li].w13) for s in sh]
        assert torch.equal(torch.cat([p[0] for p in parts]), g) and torch.equal(torch.cat([p[1] for p in parts]), u)
    assert sh[1].embed is w.embed and sh[1].lm_head is w.lm_head


def test_sharded_math_equals_the_full_forward():
    seqs = [[5, 9, 200, 17], list(range(3, 90, 2))]
    cfg4 = LlamaConfig(vocab_size=1024, hidden=512, layers=2, heads=8, kv_heads=4, ffn=1024, max_pos=2048)
    for cfg, world in ((CFG, 2), (cfg4, 4)):
        w = LlamaWeights.random(cfg, "cpu", seed=2, std=0.05)
        for a, b in zip(reference_tp_forward(w, seqs, world), reference_forward(w, seqs)):
            assert torch.allclose(a, b, atol=1e-3, rtol=1e-3), (world, (a - b).abs().max().item())


def test_shapes_that_do_not_split_are_refused():
    with pytest.raises(ValueError):
        tp_config(CFG, 3)                               # 8 heads / 2 KV heads
    with pytest.raises(ValueError):
        tp_config(LlamaConfig(ffn=640), 2)              # 320 rows per rank: not whole 128-row blocks


def _rank(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from connex_b200.models import llama as L

        def gemm(a, b, out, residual=None, status=None, **kw):     # the GEMM's epilogues, on the CPU
            r = a.float() @ b.float().t()
            if residual is not None:
                r = r + residual.float()
            out.copy_(r.to(out.dtype))
            return out
        L.ops.gemm = gemm
        g = torch.Generator().manual_seed(5)
        a_full = torch.randn(3, 64, generator=g)
        w_full = torch.randn(32, 64, generator=g)
        x0 = torch.randn(3, 32, generator=g)
        model = L.LlamaModel.__new__(L.LlamaModel)
        model.tp, model.status = TPGroup(rank, 2), None
        x = x0.clone()
        # row-parallel: this rank holds its half of the input columns
        model._residual_gemm(a_full[:, rank * 32:(rank + 1) * 32], w_full[:, rank * 32:(rank + 1) * 32], x)
        q.put((rank, torch.allclose(x, x0 + a_full @ w_full.t(), atol=1e-4)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_row_parallel_all_reduce_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(30)
    assert res == {0: True, 1: True}, res


def _gpu_rank(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
        from connex_b200.models.llama import LlamaModel, PagedKVCache, slot_mapping
        w = LlamaWeights.random(CFG, dev, seed=4)
        sh = shard_llama(w, rank, 2)
        cache = PagedKVCache(sh.cfg, 64, dev)
        model = LlamaModel(sh, cache, max_tokens=1024, max_batch=4, tp=TPGroup(rank, 2))
        seqs = [[5, 9, 200], list(range(3, 300, 3))]
        ids, pos, slots, rows, r = [], [], [], [], 0
        for s in seqs:
            blocks = cache.allocate(cache.blocks_needed(len(s)))
            ids += s
            pos += list(range(len(s)))
            slots += slot_mapping(blocks, 0, len(s), CFG.block_size)
            r += len(s)
            rows.append(r - 1)
        t = lambda x, dt: torch.tensor(x, dtype=dt, device=dev)
        nxt = model.prefill(t(ids, torch.int32), t(pos, torch.int32), t(slots, torch.int64), [len(s) for s in seqs],
                            t(rows, torch.int32), ops.prefill_tile_info([len(s) for s in seqs], dev)).tolist()
        ok = True
        for s, tok, lg in zip(seqs, nxt, reference_forward(w, seqs)):
            top = lg.max().item()
            ok &= lg[int(tok)].item() >= top - 0.05 * (abs(top) + 1)
        q.put((rank, (bool(ok), nxt)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.gpu
def test_two_gpu_tensor_parallel_prefill():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_gpu_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(60)
    assert all(isinstance(v, tuple) and v[0] for v in res.values()), res
    assert res[0][1] == res[1][1]                        # the ranks agree on every token

"""Pipeline runtime on one B200: a model split in two stages (separate
weights, caches and the residual stream handed over) gives the same greedy
tokens as the unsplit model, for prefill and for decode."""
import pytest
import torch

from connex.pp.handover import CX_CTX, REQUEST_IDS

pytestmark = pytest.mark.gpu


def test_two_stage_split_matches_whole_model():
    from connex_b200 import ops
    from connex_b200.models.llama import LlamaConfig, LlamaModel, LlamaWeights, PagedKVCache
    from connex_b200.runtime.pp import StageRuntime
    dev = torch.device("cuda", 0)
    cfg = LlamaConfig.tiny(layers=4)
    s0 = StageRuntime(cfg, 0, 2, dev, num_blocks=256, max_tokens=2048, max_batch=8, max_ctx=512)
    s0.enable_activation_log(8)
    s1 = StageRuntime(cfg, 2, 4, dev, num_blocks=256, max_tokens=2048, max_batch=8, max_ctx=512)
    whole = LlamaWeights(cfg=cfg, embed=s0.weights.embed, layers=s0.weights.layers + s1.weights.layers,
                         final_norm=s1.weights.final_norm, lm_head=s1.weights.lm_head)
    cache = PagedKVCache(cfg, 256, dev)
    model = LlamaModel(whole, cache, 2048, 8)
    lens = [100, 37, 64]
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    rids = ["a", "b", "c"]
    ids = torch.tensor(sum(seqs, []), dtype=torch.int32, device=dev)
    td = {"kind": "prefill", REQUEST_IDS: rids, CX_CTX: [0, 0, 0], "n_new": lens, "ids": ids}
    x = s0.compute(td, [])["x"]
    nxt = s1.compute({**td, "x": x}, [])["next"]
    # whole model on the same prompts
    tables = [cache.allocate(cache.blocks_needed(n + 8)) for n in lens]
    from connex_b200.models.llama import slot_mapping
    slots = torch.tensor(sum((slot_mapping(t, 0, n, 16) for t, n in zip(tables, lens)), []), dtype=torch.int64,
                         device=dev)
    pos = torch.tensor(sum((list(range(n)) for n in lens), []), dtype=torch.int32, device=dev)
    last = torch.tensor([sum(lens[:i + 1]) - 1 for i in range(3)], dtype=torch.int32, device=dev)
    want = model.prefill(ids, pos, slots, lens, last, ops.prefill_tile_info(lens, dev))
    torch.cuda.synchronize()
    assert nxt.tolist() == want.tolist()
    # two decode steps through the split pipeline vs the whole model
    cur = want.clone()
    ctx = list(lens)
    for _ in range(2):
        td = {"kind": "decode", REQUEST_IDS: rids, CX_CTX: ctx, "n_new": [1, 1, 1], "ids": cur.to(torch.int32)}
        x = s0.compute(td, [])["x"]
        got = s1.compute({**td, "x": x}, [])["next"]
        bt = torch.zeros(3, 8, dtype=torch.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        dslots = torch.tensor([slot_mapping(t, c, 1, 16)[0] for t, c in zip(tables, ctx)], dtype=torch.int64,
                              device=dev)
        ws = ops.decode_workspace(3, cfg.heads, 512, dev)
        ref = model.decode(cur.to(torch.int32), torch.tensor(ctx, dtype=torch.int32, device=dev), dslots,
                           bt.to(dev), torch.tensor([c + 1 for c in ctx], dtype=torch.int32, device=dev),
                           max(ctx) + 1, ws, torch.arange(3, dtype=torch.int32, device=dev))
        torch.cuda.synchronize()
        assert got.tolist() == ref.tolist()
        cur = ref.clone()
        ctx = [c + 1 for c in ctx]
    # failover: a fresh replica of stage 1 is refilled from stage 0's logged outputs (no stage-0
    # recompute) and then predicts exactly what the old replica would have
    s1b = StageRuntime(cfg, 2, 4, dev, num_blocks=256, max_tokens=2048, max_batch=8, max_ctx=512)
    x, lens2 = s0.replay(rids)
    assert lens2 == ctx
    nb = s1b.compute({"kind": "prefill", REQUEST_IDS: rids, CX_CTX: [0, 0, 0], "n_new": lens2, "x": x}, [])["next"]
    torch.cuda.synchronize()
    assert nb.tolist() == cur.tolist()
    # a stage that lost a request's KV reports it and does not claim it
    td = {"kind": "decode", REQUEST_IDS: ["zz"], CX_CTX: [40], "n_new": [1], "ids": cur[:1].to(torch.int32)}
    s0.compute(td, ["zz"])
    assert s0.kv_held("zz") == 0

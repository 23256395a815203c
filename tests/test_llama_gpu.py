"""Llama runtime on the native kernels vs the fp32 PyTorch forward."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(layers=2, num_blocks=256, seed=0):
    from connex_b200.models.llama import LlamaConfig, LlamaModel, LlamaWeights, PagedKVCache
    dev = torch.device("cuda", 0)
    cfg = LlamaConfig.tiny(layers=layers)
    w = LlamaWeights.random(cfg, dev, seed=seed)
    cache = PagedKVCache(cfg, num_blocks, dev)
    return cfg, w, cache, LlamaModel(w, cache, max_tokens=4096, max_batch=16)


def _prefill(model, cache, seqs):
    from connex_b200 import ops
    from connex_b200.models.llama import slot_mapping
    dev = model.device
    ids, pos, slots, rows, tables = [], [], [], [], []
    r = 0
    for s in seqs:
        blocks = cache.allocate(cache.blocks_needed(len(s) + 8))
        tables.append(blocks)
        ids += s
        pos += list(range(len(s)))
        slots += slot_mapping(blocks, 0, len(s), cache.cfg.block_size)
        r += len(s)
        rows.append(r - 1)
    t = lambda x, dt: torch.tensor(x, dtype=dt, device=dev)
    out = model.prefill(t(ids, torch.int32), t(pos, torch.int32), t(slots, torch.int64),
                        [len(s) for s in seqs], t(rows, torch.int32),
                        ops.prefill_tile_info([len(s) for s in seqs], dev))
    return out.clone(), tables


def test_prefill_matches_reference():
    from connex_b200.models.llama import reference_forward
    cfg, w, cache, model = _setup()
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 70, 200)]
    nxt, _ = _prefill(model, cache, seqs)
    ref = reference_forward(w, seqs)
    for i, lg in enumerate(ref):
        # the kernel's greedy token must be (near-)argmax of the fp32 logits
        top = lg.max().item()
        assert lg[int(nxt[i])].item() >= top - 0.05 * (abs(top) + 1), (i, int(nxt[i]), int(lg.argmax()))


def test_decode_matches_prefill():
    """prefill(n) + decode(1 token) gives the same next token as prefill(n+1)."""
    from connex_b200 import ops
    from connex_b200.models.llama import slot_mapping, reference_forward
    cfg, w, cache, model = _setup()
    g = torch.Generator().manual_seed(1)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 31, 130)]
    nxt, tables = _prefill(model, cache, seqs)
    dev = model.device
    B = len(seqs)
    maxb = max(len(t) for t in tables)
    bt = torch.tensor([t + [0] * (maxb - len(t)) for t in tables], dtype=torch.int32, device=dev)
    pos = torch.tensor([len(s) for s in seqs], dtype=torch.int32, device=dev)
    slots = torch.tensor([slot_mapping(t, len(s), 1, cfg.block_size)[0] for t, s in zip(tables, seqs)],
                         dtype=torch.int64, device=dev)
    ctx = pos + 1
    ws = ops.decode_workspace(B, cfg.heads, int(ctx.max()), dev)
    rows = torch.arange(B, dtype=torch.int32, device=dev)
    dec = model.decode(nxt, pos, slots, bt, ctx, int(ctx.max()), ws, rows).clone()
    ref = reference_forward(w, [s + [int(t)] for s, t in zip(seqs, nxt.tolist())])
    for i, lg in enumerate(ref):
        top = lg.max().item()
        assert lg[int(dec[i])].item() >= top - 0.05 * (abs(top) + 1)

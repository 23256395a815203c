"""Hugging Face Llama checkpoints: the loader's fused layouts reproduce
``transformers``' ``LlamaForCausalLM`` logits in fp32 (grouped-query heads,
Llama 3.1 RoPE scaling, tied embeddings), a pipeline stage reads only its
layers, ``save_llama`` round-trips, unsupported configs are refused, and on
a GPU the native kernels' greedy tokens on a loaded checkpoint are the
(near-)argmax of the transformers logits."""
import json

import pytest
import torch

from connex_b200.models.hf import config_from_hf, load_llama, save_llama
from connex_b200.models.llama import LlamaConfig, LlamaWeights, reference_forward

transformers = pytest.importorskip("transformers")

SCALING = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
           "original_max_position_embeddings": 64}


def _hf_model(path, tie=False, scaling=True, layers=2, seed=0, **shape):
    torch.manual_seed(seed)
    geo = dict(vocab_size=512, hidden_size=256, num_attention_heads=2, num_key_value_heads=1, intermediate_size=256)
    geo.update(shape)
    hc = transformers.LlamaConfig(num_hidden_layers=layers, head_dim=128, rope_theta=500000.0,
                                  max_position_embeddings=1024, rms_norm_eps=1e-5, tie_word_embeddings=tie,
                                  rope_scaling=dict(SCALING) if scaling else None, **geo)
    m = transformers.LlamaForCausalLM(hc).float().eval()
    with torch.no_grad():                       # non-trivial norms so a swapped norm tensor shows
        for n, p in m.named_parameters():
            if "norm" in n:
                p.uniform_(0.5, 1.5)
    m.save_pretrained(str(path))
    return m


def _hf_logits(m, seq):
    with torch.no_grad():
        return m(torch.tensor([seq])).logits[0, -1]


@pytest.mark.parametrize("tie,scaling", [(False, True), (True, False)])
def test_loaded_weights_match_transformers(tmp_path, tie, scaling):
    m = _hf_model(tmp_path, tie=tie, scaling=scaling)
    w = load_llama(str(tmp_path), "cpu", dtype=torch.float32)
    assert (w.cfg.rope_scaling is not None) == scaling
    if tie:
        assert w.lm_head is w.embed
    for seq in ([5, 9, 200], list(range(3, 300, 3))):         # 99 positions: past the original 64 context
        ref = reference_forward(w, [seq])[0]
        hf = _hf_logits(m, seq)
        assert torch.allclose(ref, hf, atol=1e-4, rtol=1e-4), (ref - hf).abs().max().item()


def test_stage_reads_only_its_layers(tmp_path):
    _hf_model(tmp_path, layers=3)
    full = load_llama(str(tmp_path), "cpu", dtype=torch.float32)
    mid = load_llama(str(tmp_path), "cpu", dtype=torch.float32, layers=(1, 2))
    last = load_llama(str(tmp_path), "cpu", dtype=torch.float32, layers=(2, 3))
    assert mid.embed is None and mid.lm_head is None and mid.final_norm is None and len(mid.layers) == 1
    assert torch.equal(mid.layers[0].wqkv, full.layers[1].wqkv) and torch.equal(mid.layers[0].w13, full.layers[1].w13)
    assert last.embed is None and torch.equal(last.lm_head, full.lm_head)
    with pytest.raises(ValueError):
        load_llama(str(tmp_path), "cpu", layers=(2, 4))


def test_save_round_trip_and_transformers_reads_it(tmp_path):
    cfg = LlamaConfig(vocab_size=512, hidden=256, layers=2, heads=2, kv_heads=1, ffn=256, max_pos=1024,
                      rope_scaling=(8.0, 1.0, 4.0, 64))
    w = LlamaWeights.random(cfg, "cpu", seed=3, std=0.05)
    save_llama(w, str(tmp_path / "ck"), max_shard_bytes=1 << 20)          # several shards + index
    idx = json.loads((tmp_path / "ck" / "model.safetensors.index.json").read_text())
    assert len(set(idx["weight_map"].values())) > 1
    back = load_llama(str(tmp_path / "ck"), "cpu")
    assert back.cfg == cfg
    for (n, a), (_, b) in zip(w.named_tensors(), back.named_tensors()):
        assert torch.equal(a, b), n
    m = transformers.LlamaForCausalLM.from_pretrained(str(tmp_path / "ck"), dtype=torch.float32).eval()
    seq = list(range(7, 400, 5))
    ref = reference_forward(back, [seq])[0]
    assert torch.allclose(ref, _hf_logits(m, seq), atol=2e-3, rtol=2e-3)


def test_unsupported_configs_are_refused():
    base = {"vocab_size": 512, "hidden_size": 256, "num_hidden_layers": 2, "num_attention_heads": 2,
            "num_key_value_heads": 1, "head_dim": 128, "intermediate_size": 256}
    assert config_from_hf(base).head_dim == 128
    for bad in ({"head_dim": 64}, {"intermediate_size": 200}, {"attention_bias": True},
                {"rope_scaling": {"rope_type": "yarn", "factor": 4.0}}):
        with pytest.raises(ValueError):
            config_from_hf({**base, **bad})
    assert config_from_hf({**base, "rope_parameters": {"rope_type": "default", "rope_theta": 1e6}}).rope_theta == 1e6


@pytest.mark.gpu
def test_native_kernels_on_a_loaded_checkpoint(tmp_path):
    from connex_b200 import ops
    from connex_b200.models.llama import LlamaModel, PagedKVCache, slot_mapping
    # the geometry of the runtime's tiny test config (hidden 512, 8 x 128 query heads, 2 KV heads)
    m = _hf_model(tmp_path, vocab_size=1024, hidden_size=512, num_attention_heads=8, num_key_value_heads=2,
                  intermediate_size=1024)
    dev = torch.device("cuda", 0)
    w = load_llama(str(tmp_path), dev)
    cache = PagedKVCache(w.cfg, 64, dev)
    model = LlamaModel(w, cache, max_tokens=1024, max_batch=4)
    seqs = [[5, 9, 200], list(range(3, 300, 3))]
    ids, pos, slots, rows, r = [], [], [], [], 0
    for s in seqs:
        blocks = cache.allocate(cache.blocks_needed(len(s)))
        ids += s
        pos += list(range(len(s)))
        slots += slot_mapping(blocks, 0, len(s), w.cfg.block_size)
        r += len(s)
        rows.append(r - 1)
    t = lambda x, dt: torch.tensor(x, dtype=dt, device=dev)
    nxt = model.prefill(t(ids, torch.int32), t(pos, torch.int32), t(slots, torch.int64), [len(s) for s in seqs],
                        t(rows, torch.int32), ops.prefill_tile_info([len(s) for s in seqs], dev)).tolist()
    for s, tok in zip(seqs, nxt):
        lg = _hf_logits(m, s)
        top = lg.max().item()
        assert lg[int(tok)].item() >= top - 0.05 * (abs(top) + 1), (int(tok), int(lg.argmax()))


def test_tensor_parallel_load_is_the_shard_of_the_full_load(tmp_path):
    from connex_b200.parallel.tp import shard_llama
    _hf_model(tmp_path, vocab_size=1024, hidden_size=512, num_attention_heads=8, num_key_value_heads=2,
              intermediate_size=1024, tie=True)
    full = load_llama(str(tmp_path), "cpu")
    for rank in range(2):
        part = load_llama(str(tmp_path), "cpu", tp=(rank, 2))
        ref = shard_llama(full, rank, 2)
        assert part.cfg == ref.cfg and part.lm_head is part.embed
        for (n, a), (_, b) in zip(part.named_tensors(), ref.named_tensors()):
            assert torch.equal(a, b), n

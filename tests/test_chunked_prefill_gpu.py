"""Chunked prefill on the GPU: the paged variant of the tcgen05 prefill
attention against its fp32 re-statement (chunks continuing cached
sequences, GQA 4 and 1, a context spanning many key tiles, one-token and
ragged chunks), and a stage runtime that reads a prompt in chunks -- with a
decode row of another request in the same steps -- producing the residual
stream of a whole-prompt prefill."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rnd(*shape, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn(*shape, generator=g, device=dev).to(torch.bfloat16)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("rows", [[(0, 100)], [(64, 128)], [(1000, 300), (17, 5)], [(2000, 1), (130, 513)],
                                  [(5, 64), (0, 200), (4000, 129)], [(2048, 2048)], [(50, 300)]])
@pytest.mark.parametrize("G", [4, 1])
@pytest.mark.parametrize("tile", [256, 128])
def test_paged_prefill_attention(dev, rows, G, tile):
    from connex_b200 import ops
    from connex_b200.ops import reference as R
    Hkv, BS, NB = 2, 16, 1024
    Hq = Hkv * G
    ctx, n_new = [c for c, _ in rows], [n for _, n in rows]
    T = sum(n_new)
    kc, vc = _rnd(NB, Hkv, BS, 128, dev=dev, seed=3), _rnd(NB, Hkv, BS, 128, dev=dev, seed=4)
    # cache slots past each sequence's end hold garbage (never written): NaN must not leak into O
    kc.view(torch.int16)[-1].fill_(-1)
    vc.view(torch.int16)[-1].fill_(-1)                   # 0xFFFF = bf16 NaN in the last physical block
    maxb = max((c + n + BS - 1) // BS for c, n in rows)
    perm = torch.randperm(NB - 1, device=dev).to(torch.int32)
    bt = perm[:len(rows) * maxb].view(len(rows), maxb).contiguous()
    for b, (c, n) in enumerate(rows):                    # each sequence's last block: the NaN-filled one's
        last = (c + n - 1) // BS                         # tail past the end stays NaN after the copy below
        if (c + n) % BS:
            kc[NB - 1, :, :(c + n) % BS] = kc[bt[b, last].long(), :, :(c + n) % BS]
            vc[NB - 1, :, :(c + n) % BS] = vc[bt[b, last].long(), :, :(c + n) % BS]
            bt[b, last] = NB - 1
            break
    qkv = _rnd(T, (Hq + 2 * Hkv) * 128, dev=dev, seed=5)
    ti = ops.prefill_tile_info(n_new, dev, ctx=ctx, tile_rows=tile)
    st = ops.new_status(dev)
    out = ops.prefill_attention_paged(qkv, kc, vc, bt, ti, Hq, Hkv, status=st, tile_rows=tile)
    torch.cuda.synchronize()
    ops.check_status(st, "prefill_attention_paged")
    ref = R.paged_prefill_attention(qkv[:, :Hq * 128].view(T, Hq, 128), kc, vc, bt, ctx, n_new)
    err = (out.view(T, Hq, 128).float() - ref).abs().max().item()
    assert err <= 2e-2 + 2e-2 * ref.abs().max().item(), err


def test_stage_runtime_reads_a_prompt_in_chunks(dev):
    from connex.pp.handover import CX_CTX, REQUEST_IDS
    from connex_b200.models.llama import LlamaConfig
    from connex_b200.runtime.pp import StageRuntime
    cfg = LlamaConfig.tiny(layers=2)
    rt = StageRuntime(cfg, 0, 1, dev, num_blocks=256, max_tokens=512, max_batch=8, max_ctx=1024, seed=0)
    g = torch.Generator().manual_seed(7)
    prompt = torch.randint(3, cfg.vocab_size, (300,), generator=g).tolist()
    other = torch.randint(3, cfg.vocab_size, (40,), generator=g).tolist()

    def step(kind, rids, ctx, n_new, ids, n_dec=None):
        td = {"kind": kind, REQUEST_IDS: rids, CX_CTX: ctx, "n_new": n_new,
              "ids": torch.tensor(ids, dtype=torch.int32, device=dev)}
        if n_dec is not None:
            td["n_dec"] = n_dec
        return rt.compute(td, [])["x"].float()

    whole = step("prefill", ["w"], [0], [300], prompt)
    step("prefill", ["o"], [0], [40], other)
    got, done, k = [], 0, 0
    while done < 300:
        n = min(64, 300 - done)
        dec_tok = other[-1] if k == 0 else 5
        x = step("mixed", ["o", "c"], [40 + k, done], [1, n], [dec_tok] + prompt[done:done + n], n_dec=1)
        got.append(x[1:])                        # row 0: the decode row of "o"
        done += n
        k += 1
    chunked = torch.cat(got)
    err = (chunked - whole).abs().max().item()
    assert err <= 3e-2 * whole.abs().max().item() + 3e-2, err
    assert rt.held["c"] == 300 and rt.held["o"] == 40 + k

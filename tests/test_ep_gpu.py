"""EP MoE over peer memory (dispatch -> tcgen05 grouped GEMMs -> combine) vs fp32 PyTorch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _weights(n_slots, H, F, dev, seed=0):
    from connex_b200 import ops
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    gate = torch.randn(n_slots, F, H, generator=g, device=dev) * 0.05
    up = torch.randn(n_slots, F, H, generator=g, device=dev) * 0.05
    w13 = torch.stack([ops.interleave_gate_up(gate[i].bfloat16(), up[i].bfloat16()) for i in range(n_slots)])
    w2 = (torch.randn(n_slots, H, F, generator=g, device=dev) * 0.05).bfloat16()
    return w13.contiguous(), w2.contiguous()


def _routing(T, E, K, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    logits = torch.randn(T, E, generator=g, device=dev)
    w, idx = torch.topk(torch.softmax(logits, -1), K, dim=-1)
    return idx.to(torch.int32).contiguous(), w.float().contiguous()


def _close(out, ref):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= 2e-2 + 3e-2 * scale, f"max err {err} vs scale {scale}"


def _identity_l2p(E, dev):
    return torch.arange(E, dtype=torch.int32, device=dev).view(E, 1).contiguous(), \
        torch.ones(E, dtype=torch.int32, device=dev)


@pytest.mark.parametrize("N,S,Ts", [(1, 16, [300]), (4, 4, [37, 100, 5, 64]), (8, 2, [1, 2, 3, 4, 5, 6, 7, 200])])
def test_ep_matches_reference(N, S, Ts):
    from connex_b200 import ops
    from connex_b200.parallel.ep import EPConfig, emulated_forward, emulated_group, reference_moe
    dev = torch.device("cuda", 0)
    H, F, K = 512, 256, 4
    E = N * S
    cfg = EPConfig(n_ranks=N, slots_per_rank=S, hidden=H, ffn=F, top_k=K, max_tokens=max(Ts))
    w13, w2 = _weights(E, H, F, dev)
    layers = emulated_group(cfg, w13, w2, dev)
    l2p, cnt = _identity_l2p(E, dev)
    for step in range(2):  # two forwards: flags are cumulative epochs
        xs = [(torch.randn(T, H, device=dev) * 0.5).bfloat16() for T in Ts]
        routes = [_routing(T, E, K, dev, 10 * step + r) for r, T in enumerate(Ts)]
        ys = emulated_forward(layers, xs, [r[0] for r in routes], [r[1] for r in routes], l2p, cnt)
        torch.cuda.synchronize()
        for L in layers:
            ops.check_status(L.b.status, f"ep rank {L.rank}")
        for r in range(N):
            _close(ys[r], reference_moe(xs[r], routes[r][0], routes[r][1], w13, w2))


def test_ep_replicas_and_unroutable_expert():
    """Logical expert 0 has two physical replicas (slots 0 and 5); logical
    expert 3 has none (its rank died): its rows are dropped, not waited for."""
    from connex_b200 import ops
    from connex_b200.parallel.ep import EPConfig, emulated_forward, emulated_group, reference_moe
    dev = torch.device("cuda", 0)
    N, S, H, F, K = 2, 4, 512, 256, 2
    E = N * S
    cfg = EPConfig(N, S, H, F, K, max_tokens=128)
    w13, w2 = _weights(E, H, F, dev, seed=3)
    w13[5] = w13[0]
    w2[5] = w2[0]
    layers = emulated_group(cfg, w13, w2, dev)
    l2p = torch.full((E, 2), -1, dtype=torch.int32, device=dev)
    cnt = torch.ones(E, dtype=torch.int32, device=dev)
    for e in range(E):
        l2p[e, 0] = e
    l2p[0, 1] = 5
    cnt[0] = 2
    cnt[3] = 0
    Ts = [50, 70]
    xs = [(torch.randn(T, H, device=dev) * 0.5).bfloat16() for T in Ts]
    routes = [_routing(T, E, K, dev, 40 + r) for r, T in enumerate(Ts)]
    ys = emulated_forward(layers, xs, [r[0] for r in routes], [r[1] for r in routes], l2p, cnt)
    torch.cuda.synchronize()
    for L in layers:
        ops.check_status(L.b.status, "ep")
    for r in range(N):
        _close(ys[r], reference_moe(xs[r], routes[r][0], routes[r][1], w13, w2, l2p, cnt))


def test_ep_rank_leaves_without_rebuild():
    """Rank 2 of 3 leaves between forwards: survivors route around its slots
    and mark it dead (its peer-table column points at local sinks, wait
    targets count live ranks) and keep going on the same buffers."""
    from connex_b200 import ops
    from connex_b200.parallel.ep import EPConfig, emulated_forward, emulated_group, reference_moe
    dev = torch.device("cuda", 0)
    N, S, H, F, K = 3, 4, 512, 256, 2
    E = N * S
    cfg = EPConfig(N, S, H, F, K, max_tokens=64)
    w13, w2 = _weights(E, H, F, dev, seed=5)
    layers = emulated_group(cfg, w13, w2, dev)
    l2p, cnt = _identity_l2p(E, dev)
    Ts = [40, 64, 13]
    for step in range(2):
        xs = [(torch.randn(T, H, device=dev) * 0.5).bfloat16() for T in Ts]
        routes = [_routing(T, E, K, dev, 7 * step + r) for r, T in enumerate(Ts)]
        emulated_forward(layers, xs, [r[0] for r in routes], [r[1] for r in routes], l2p, cnt)
    torch.cuda.synchronize()
    # rank 2 dies; its experts move (here: logical experts 8..11 now served by slots 0..3 copies)
    w13s, w2s = w13.clone(), w2.clone()
    survivors = layers[:2]
    for L in survivors:
        L.mark_dead(2)
    l2p2 = l2p.clone()
    for e in range(8, 12):
        l2p2[e, 0] = e - 8 + 4          # served by rank 1's slots (weights of those slots)
    for step in range(3):
        xs = [(torch.randn(T, H, device=dev) * 0.5).bfloat16() for T in Ts[:2]]
        routes = [_routing(T, E, K, dev, 100 + 7 * step + r) for r, T in enumerate(Ts[:2])]
        ys = emulated_forward(survivors, xs, [r[0] for r in routes], [r[1] for r in routes], l2p2, cnt)
        torch.cuda.synchronize()
        for L in survivors:
            ops.check_status(L.b.status, f"ep rank {L.rank}")
        for r in range(2):
            _close(ys[r], reference_moe(xs[r], routes[r][0], routes[r][1], w13s, w2s, l2p2, cnt))

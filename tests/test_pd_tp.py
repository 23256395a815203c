"""Heterogeneous-TP KV transfer on CPU: the head plan of every (prefill TP,
decode TP) pair, head-slice reads between HND and NHD caches, and end-to-end
pulls over real ZeroMQ control with the loopback data plane where every
decode rank gathers exactly its heads from the prefill ranks; leases with
several readers, and one dead prefill rank failing the whole pull."""
import ctypes
import itertools
import time

import pytest
import torch

from connex.pd.dataplane import LoopbackPlane
from connex.pd.kv_layout import TensorLayout, head_read_ops, tp_plan
from connex.pd.transfer import KVConsumer, KVProducer

H, BS, HB, NB = 8, 16, 32, 24            # KV heads, block tokens, bytes per head and token, blocks


@pytest.mark.parametrize("local_tp,remote_tp", [(1, 1), (2, 2), (1, 4), (2, 8), (4, 1), (8, 2), (4, 8)])
def test_tp_plan_covers_every_head_exactly_once(local_tp, remote_tp):
    seen = []
    for r in range(local_tp):
        base = r * H // local_tp
        for s in tp_plan(r, local_tp, remote_tp, H):
            assert 0 <= s.remote_rank < remote_tp and s.nheads > 0
            glob_local = [base + s.local_head0 + i for i in range(s.nheads)]
            glob_remote = [s.remote_rank * H // remote_tp + s.remote_head0 + i for i in range(s.nheads)]
            assert glob_local == glob_remote                    # same global heads on both sides
            seen += glob_local
    assert sorted(seen) == list(range(H))
    # every remote rank has exactly one releaser among the local ranks that read it
    rel = {}
    for r in range(local_tp):
        for s in tp_plan(r, local_tp, remote_tp, H):
            rel.setdefault(s.remote_rank, []).append((r, s.releaser, s.readers))
    for readers in rel.values():
        assert sum(x[1] for x in readers) == 1 and all(x[2] == len(readers) for x in readers)


def test_tp_plan_shapes():
    assert [(s.remote_rank, s.nheads) for s in tp_plan(1, 2, 2, H)] == [(1, 4)]         # equal: own rank
    assert [(s.remote_rank, s.nheads) for s in tp_plan(0, 2, 4, H)] == [(0, 2), (1, 2)]  # smaller: two ranks
    shared = [tp_plan(r, 4, 2, H)[0] for r in range(4)]                                  # larger: shared
    assert [(s.remote_rank, s.remote_head0, s.readers, s.releaser) for s in shared] == \
        [(0, 0, 2, True), (0, 2, 2, False), (1, 0, 2, True), (1, 2, 2, False)]
    with pytest.raises(ValueError, match="replicated"):
        tp_plan(0, 16, 1, H)                                   # 8 heads over 16 ranks would replicate
    with pytest.raises(ValueError):
        tp_plan(2, 2, 1, H)


def _cache(heads: int, hnd: bool):
    """A [2, NB, ...] KV cache of ``heads`` heads and its layout."""
    shape = (2, NB, heads, BS, HB) if hnd else (2, NB, BS, heads, HB)
    t = torch.zeros(shape, dtype=torch.uint8)
    lo = TensorLayout(base=t.data_ptr(), outer=2, outer_stride=t.stride(0), block_stride=t.stride(1),
                      seg_bytes=t.stride(1), num_blocks=NB)
    lo = lo.with_heads(heads, BS * HB if hnd else HB, BS, HB if hnd else heads * HB, HB)
    return t, lo


def _heads(t, hnd: bool):
    """[2, NB, heads, BS, HB] view whatever the layout."""
    return t if hnd else t.permute(0, 1, 3, 2, 4)


def test_head_read_ops_between_hnd_and_nhd():
    src, slo = _cache(8, hnd=True)
    src.copy_(torch.randint(0, 255, src.shape, dtype=torch.uint8))
    for hnd in (True, False):
        dst, dlo = _cache(4, hnd)
        ops = head_read_ops([dlo], [slo], [5], [9], 0, 4, 4)          # remote heads 4..7 -> local 0..3
        for d, s, n in ops:
            ctypes.memmove(d, s, n)
        assert torch.equal(_heads(dst, hnd)[:, 5], src[:, 9, 4:8])
        if hnd:
            assert len(ops) == 2                                       # one read per K / V segment
    with pytest.raises(ValueError, match="outside"):
        head_read_ops([dlo], [slo], [0], [0], 2, 6, 4)


@pytest.mark.parametrize("p_tp,d_tp,p_hnd,d_hnd", [
    (1, 2, True, True), (2, 1, True, False), (2, 4, False, True), (4, 2, True, True), (2, 2, False, False)])
def test_heterogeneous_tp_pull_gathers_each_ranks_heads(p_tp, d_tp, p_hnd, d_hnd):
    g = torch.Generator().manual_seed(p_tp * 10 + d_tp)
    full = torch.randint(0, 255, (2, NB, H, BS, HB), dtype=torch.uint8, generator=g)
    src_blocks, dst_blocks = [3, 4, 7], [10, 11, 20]
    prods, caches = [], []
    try:
        for p in range(p_tp):
            t, lo = _cache(H // p_tp, p_hnd)
            _heads(t, p_hnd).copy_(full[:, :, p * H // p_tp:(p + 1) * H // p_tp])
            pr = KVProducer(LoopbackPlane(), [lo], bind_ip="127.0.0.1", retain_s=30)
            pr.hold("r", "tid", src_blocks)
            prods.append(pr)
            caches.append(t)
        addrs = [f"127.0.0.1:{pr.port}" for pr in prods]
        for d in range(d_tp):
            t, lo = _cache(H // d_tp, d_hnd)
            cons = KVConsumer(LoopbackPlane(), [lo], release_after_pull=True, who=f"d{d}")
            try:
                srcs = [(addrs[s.remote_rank], s) for s in tp_plan(d, d_tp, p_tp, H)]
                cons.pull("r", addrs[0], "tid", dst_blocks, sources=srcs)
                res = _wait(cons)
                assert res.ok, res.why
                mine = _heads(t, d_hnd)
                for lb, rb in zip(dst_blocks, src_blocks):
                    assert torch.equal(mine[:, lb], full[:, rb, d * H // d_tp:(d + 1) * H // d_tp])
            finally:
                cons.close()
        # every prefill rank was released by all of its readers: every hold is gone
        assert all(pr.held() == 0 for pr in prods)
    finally:
        for pr in prods:
            pr.close()


def _wait(cons, timeout=5.0):
    deadline = time.time() + timeout
    while time.time() < deadline:
        done = cons.take_done()
        if done:
            return done[0]
        time.sleep(0.005)
    raise AssertionError("pull did not finish")


def test_hold_is_freed_only_after_every_reader_released():
    t, lo = _cache(8, True)
    pr = KVProducer(LoopbackPlane(), [lo], bind_ip="127.0.0.1", retain_s=30)
    try:
        pr.hold("r", "tid", [1, 2])
        src = tp_plan(0, 2, 1, H)[0]                         # two decode ranks read prefill rank 0
        addr = f"127.0.0.1:{pr.port}"
        for who, expect in (("a", 1), ("b", 0)):
            dt, dlo = _cache(4, True)
            cons = KVConsumer(LoopbackPlane(), [dlo], release_after_pull=True, who=who)
            try:
                cons.pull("r", addr, "tid", [5, 6], sources=[(addr, src)])
                assert _wait(cons).ok
                deadline = time.time() + 2
                while pr.held() != expect and time.time() < deadline:
                    time.sleep(0.01)
                assert pr.held() == expect
            finally:
                cons.close()
        assert "r" in pr.take_finished()
    finally:
        pr.close()


def test_one_dead_prefill_rank_fails_the_whole_pull():
    prods = []
    for p in range(2):
        t, lo = _cache(4, True)
        pr = KVProducer(LoopbackPlane(), [lo], bind_ip="127.0.0.1", retain_s=30)
        pr.hold("r", "tid", [1])
        prods.append((pr, t))
    addrs = [f"127.0.0.1:{pr.port}" for pr, _ in prods]
    prods[1][0].close()                                      # prefill rank 1 is gone
    dt, dlo = _cache(8, True)
    cons = KVConsumer(LoopbackPlane(), [dlo], ctrl_timeout_ms=200, acquire_wait_s=0.2)
    try:
        cons.pull("r", addrs[0], "tid", [3], sources=[(addrs[s.remote_rank], s) for s in tp_plan(0, 1, 2, H)])
        res = _wait(cons)
        assert not res.ok and "TP rank 1" in res.why and res.failed_blocks == [3]
    finally:
        cons.close()
        prods[0][0].close()


def test_plans_for_every_power_of_two_pair_are_consistent():
    for lt, rt in itertools.product([1, 2, 4, 8], repeat=2):
        total = sum(s.nheads for r in range(lt) for s in tp_plan(r, lt, rt, H))
        assert total == H

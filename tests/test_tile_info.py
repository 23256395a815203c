"""Prefill attention work lists (CPU): ``prefill_tile_info`` lists every
(sequence, first query) tile exactly once, heaviest first (query rows x keys
attended), for both tile sizes and with cached context (chunked prefill)."""
import pytest
import torch

from connex_b200 import ops


def _expected(seq_lens, ctx, step):
    rows, start = [], 0
    for i, n in enumerate(seq_lens):
        for q0 in range(0, n, step):
            rows.append((start, n, q0) if ctx is None else (start, n, q0, ctx[i], i))
        start += n
    return rows


def _work(row, step):
    start, n, q0 = row[:3]
    c = row[3] if len(row) > 3 else 0
    r = min(step, n - q0)
    return r * (c + q0 + r / 2)


@pytest.mark.parametrize("tile", [128, 256])
@pytest.mark.parametrize("ctx", [None, [0, 4096, 17, 300]])
def test_every_tile_once_heaviest_first(tile, ctx):
    lens = [2048, 130, 1, 700]
    got = [tuple(r) for r in ops.prefill_tile_info(lens, "cpu", ctx=ctx, tile_rows=tile).tolist()]
    want = _expected(lens, ctx, tile)
    assert sorted(got) == sorted(want)
    works = [_work(r, tile) for r in got]
    assert works == sorted(works, reverse=True)


def test_empty_batch():
    t = ops.prefill_tile_info([], "cpu")
    assert t.shape == (0, 3) and t.dtype == torch.int32

"""Python surface of the sm_100a kernels in ``connex_b200._C``.

Every function here launches one of this package's own CUDA kernels on the
current torch stream.  There is no fallback: if the extension is missing the
import of :mod:`connex_b200.ops` raises, so a GPU run can never silently
execute a PyTorch re-statement instead of the native kernels.  (The fp32
PyTorch re-statements used as test oracles live in
:mod:`connex_b200.ops.reference` and are never called from here.)
"""
from __future__ import annotations

import math
from typing import Optional

import torch

try:
    from connex_b200 import _C  # noqa: F401
except ImportError as e:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "connex_b200._C is not built; run `python setup.py build_ext --inplace` "
        f"(sm_100a) before using connex_b200.ops: {e}") from e

EPI_STORE = _C.EPI_STORE
EPI_ADD = _C.EPI_ADD
EPI_SILU_MUL = _C.EPI_SILU_MUL

# Tile width of the fused SiLU(gate)*up epilogue: weights for it are stored
# with gate and up rows interleaved in blocks of GATE_UP_TILE // 2.
GATE_UP_TILE = 256


_LAUNCHES = [0]


def launch_count() -> int:
    """Number of this package's kernel launches issued so far by this process."""
    return _LAUNCHES[0]


def _n(k: int = 1) -> None:
    _LAUNCHES[0] += k


def new_status(device) -> torch.Tensor:
    """An int32 device status word (0 = ok) that kernels write error codes to."""
    return torch.zeros(1, dtype=torch.int32, device=device)


STATUS_NAMES = {0: "ok", 1: "timeout", 2: "bounds", 3: "peer-abort"}


def check_status(status: torch.Tensor, what: str = "kernel") -> None:
    code = int(status.item())
    if code != 0:
        raise RuntimeError(f"{what}: device status {code} ({STATUS_NAMES.get(code, '?')})")


# ----------------------------------------------------------------- GEMM
_SPLIT_WS: dict = {}


_SPLIT_WS_RETIRED: list = []


def _split_workspace(device, n: int) -> torch.Tensor:
    """Per-device fp32 split-K workspace; the finalize kernel leaves it zero.

    A workspace that is outgrown is kept alive, not freed: CUDA graphs that
    captured GEMMs hold its address (and it stays zero between uses)."""
    ws = _SPLIT_WS.get(device)
    if ws is None or ws.numel() < n:
        if ws is not None:
            _SPLIT_WS_RETIRED.append(ws)
        ws = torch.zeros(max(n, 1 << 20, 2 * ws.numel() if ws is not None else 0), dtype=torch.float32,
                         device=device)
        _SPLIT_WS[device] = ws
    return ws


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, *,
         residual: Optional[torch.Tensor] = None, silu_mul: bool = False, bn: int = 0,
         status: Optional[torch.Tensor] = None, max_ctas: int = 0, splits: Optional[int] = None) -> torch.Tensor:
    """``a[M,K] @ b[N,K]^T`` on tcgen05 tensor cores (bf16 in/out, fp32 accumulate).

    ``residual`` adds a bf16 tensor in the epilogue (may alias ``out``).
    ``silu_mul`` treats ``b`` as gate/up rows interleaved per 256-row tile
    (see :func:`interleave_gate_up`) and writes ``SiLU(gate) * up`` of width N/2.
    ``splits`` cuts the K loop for small-M GEMMs (None: the kernel's choice,
    1: never); a split GEMM is two launches (MMA + finalize).
    """
    M, N, K = a.shape[0], b.shape[0], a.shape[1]
    if out is None:
        out = torch.empty(M, N // 2 if silu_mul else N, dtype=torch.bfloat16, device=a.device)
    epi = EPI_SILU_MUL if silu_mul else (EPI_ADD if residual is not None else EPI_STORE)
    s = _C.gemm_splits(M, N, K, epi, bn) if splits is None else splits
    ws = _split_workspace(a.device, M * N) if s > 1 else None
    _C.gemm(a, b, out, residual, epi, bn, status, max_ctas, ws, s)
    _n(2 if s > 1 else 1)
    return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, tile: int = GATE_UP_TILE) -> torch.Tensor:
    """Stack gate [F,K] and up [F,K] as [2F,K] with rows interleaved in blocks
    of tile/2, the weight layout of the fused SiLU-mul GEMM epilogue."""
    F, K = gate.shape
    half = tile // 2
    assert F % half == 0, "FFN width must be a multiple of half the tile"
    g = gate.reshape(F // half, half, K)
    u = up.reshape(F // half, half, K)
    return torch.stack([g, u], dim=1).reshape(2 * F, K).contiguous()


def deinterleave_gate_up(w: torch.Tensor, tile: int = GATE_UP_TILE):
    F2, K = w.shape
    half = tile // 2
    x = w.reshape(F2 // tile, 2, half, K)
    return x[:, 0].reshape(-1, K), x[:, 1].reshape(-1, K)


# ------------------------------------------------------------- layers
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm of ``x`` (or of ``x + residual``, written back into ``residual``)."""
    if out is None:
        out = torch.empty_like(x)
    _C.rmsnorm(x, residual, weight, out, eps)
    _n()
    return out


def rope_cache(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, n_q_heads: int,
               n_kv_heads: int, slot_mapping: Optional[torch.Tensor] = None,
               k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
               status: Optional[torch.Tensor] = None, q_norm: Optional[torch.Tensor] = None,
               k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6) -> None:
    """Rotate q/k of the fused QKV rows in place; write k/v to their paged slots.
    ``q_norm`` / ``k_norm`` ([128] bf16): per-head RMSNorm of q / k first (Qwen3)."""
    _C.rope_cache(qkv, positions, cos_sin, slot_mapping, k_cache, v_cache, n_q_heads, n_kv_heads, status, q_norm,
                  k_norm, eps)
    _n()


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, device, scaling=None) -> torch.Tensor:
    """fp32 [max_pos, head_dim] table: cos in the first half, sin in the second.

    ``scaling = (factor, low_freq_factor, high_freq_factor, original_max_pos)``
    applies the Llama 3.1 long-context frequency rule: wavelengths shorter
    than ``original_max_pos / high_freq_factor`` keep their frequency, those
    longer than ``original_max_pos / low_freq_factor`` are divided by
    ``factor``, and the band between blends the two linearly in
    ``original_max_pos / wavelength``."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling is not None:
        factor, lo, hi, orig = (float(v) for v in scaling)
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        blended = (1 - smooth) * inv / factor + smooth * inv
        inv = torch.where(wavelen < orig / hi, inv, torch.where(wavelen > orig / lo, inv / factor, blended))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).to(torch.float32).to(device)


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None,
              status: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    _C.embedding(ids, table, out, status)
    _n()
    return out


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _C.argmax(logits, out)
    _n()
    return out


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(idx.numel(), src.shape[1], dtype=src.dtype, device=src.device)
    _C.gather_rows(src, idx, out)
    _n()
    return out


# ---------------------------------------------------------- attention
# Query rows per work item of the prefill attention: 256 runs the persistent
# kernel with two 128-row tiles per CTA (one CTA per SM; measured faster on
# 8 x 2048, 2 x 8192 and the paged chunk case), 128 the one-tile kernel (two
# CTAs per SM).  ``prefill_tile_info`` and the attention calls take the same
# ``tile_rows`` (both default to this).
PREFILL_TILE = 256


def prefill_tile_info(seq_lens, device, ctx=None, tile_rows: Optional[int] = None) -> torch.Tensor:
    """[n_tiles, 3] int32 (seq start row, seq length, first query of the tile);
    with ``ctx`` (tokens already in the cache per sequence, chunked prefill)
    [n_tiles, 5] adding (context length, sequence index) for the paged kernel.
    Rows are ordered by work, heaviest first (query rows x keys they attend
    to): the kernels hand them out in that order, so the last wave holds the
    lightest tiles."""
    step = tile_rows or PREFILL_TILE
    rows, work = [], []
    start = 0
    for i, n in enumerate(seq_lens):
        c = 0 if ctx is None else int(ctx[i])
        for q0 in range(0, n, step):
            rows.append((start, n, q0) if ctx is None else (start, n, q0, c, i))
            r = min(step, n - q0)
            work.append(r * (c + q0 + r / 2))
        start += n
    rows = [rows[k] for k in sorted(range(len(rows)), key=lambda k: -work[k])]
    width = 3 if ctx is None else 5
    t = torch.tensor(rows if rows else [(0,) * width], dtype=torch.int32)
    if not rows:
        return t[:0].to(device)
    return t.pin_memory().to(device, non_blocking=True) if torch.cuda.is_available() else t.to(device)


def prefill_attention(qkv: torch.Tensor, tile_info: torch.Tensor, n_q_heads: int, n_kv_heads: int,
                      out: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                      status: Optional[torch.Tensor] = None, tile_rows: Optional[int] = None) -> torch.Tensor:
    """Causal varlen prefill attention on the tcgen05 tensor cores.  ``qkv``
    is the fused [T, (Hq + 2 Hkv) * 128] projection output; ``tile_info``
    from ``prefill_tile_info`` with the same ``tile_rows``."""
    if out is None:
        out = torch.empty(qkv.shape[0], n_q_heads * 128, dtype=qkv.dtype, device=qkv.device)
    _C.prefill_attention(qkv, out, tile_info, n_q_heads, n_kv_heads,
                         scale if scale is not None else 1.0 / math.sqrt(128), status, tile_rows or PREFILL_TILE)
    _n()
    return out


def prefill_attention_paged(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, tile_info: torch.Tensor, n_q_heads: int, n_kv_heads: int,
                            out: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                            status: Optional[torch.Tensor] = None,
                            tile_rows: Optional[int] = None) -> torch.Tensor:
    """Causal prefill attention of chunks that continue cached sequences (the
    tcgen05 kernel's paged variant): queries from ``qkv``, keys and values of
    the whole context -- this chunk's included, already written to the cache
    -- from ``k_cache`` / ``v_cache`` [blocks, Hkv, 16, 128] through
    ``block_tables`` [B, max_blocks]; ``tile_info`` from
    ``prefill_tile_info(n_new, device, ctx)``."""
    if out is None:
        out = torch.empty(qkv.shape[0], n_q_heads * 128, dtype=qkv.dtype, device=qkv.device)
    _C.prefill_attention_paged(qkv, k_cache, v_cache, block_tables, out, tile_info, n_q_heads, n_kv_heads,
                               scale if scale is not None else 1.0 / math.sqrt(128), status,
                               tile_rows or PREFILL_TILE)
    _n()
    return out


def decode_workspace(batch: int, n_q_heads: int, max_ctx: int, device) -> torch.Tensor:
    return torch.empty(_C.decode_workspace_floats(batch, n_q_heads, max_ctx), dtype=torch.float32,
                       device=device)


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     block_tables: torch.Tensor, ctx_lens: torch.Tensor, n_q_heads: int, max_ctx: int,
                     workspace: torch.Tensor, out: Optional[torch.Tensor] = None,
                     scale: Optional[float] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(q.shape[0], n_q_heads * 128, dtype=q.dtype, device=q.device)
    _C.decode_attention(q, k_cache, v_cache, block_tables, ctx_lens, out, n_q_heads, max_ctx,
                        scale if scale is not None else 1.0 / math.sqrt(128), workspace)
    splits = _C.decode_attention_plan(q.shape[0], n_q_heads, k_cache.shape[1], max_ctx, workspace.numel())
    _n(1 if splits == 1 else 2)
    return out


# ------------------------------------------------------- peer memory
def kv_push_layer(src_k: int, src_v: int, dst_k: int, dst_v: int, pairs: torch.Tensor, *,
                  src_heads: int, dst_heads: int, src_h0: int = 0, dst_h0: int = 0,
                  n_heads: Optional[int] = None, chunk_bytes: int, src_blocks: int, dst_blocks: int,
                  ready: int = 0, max_ctas: int = 0, status: Optional[torch.Tensor] = None,
                  span: int = 0, threads: int = 256) -> int:
    """Push one layer's paged KV blocks (pairs: int32 [n, 2] of src/dst block
    ids) from local caches to (peer-mapped) destination caches.  Returns the
    number of CTAs, each of which adds 1 to the u32 at ``ready`` when done.
    ``span``: address of two int64 set to (-1, 0); the kernel stores its
    execution window there (``%globaltimer`` ns of the first CTA's start and
    the last CTA's end).  ``threads`` per CTA: 256, or 128 for a push beside
    the prefill's persistent kernels (one such CTA fits on each SM next to
    them)."""
    _n()
    return _C.kv_push_layer(src_k, src_v, dst_k, dst_v, pairs, src_heads, dst_heads, src_h0, dst_h0,
                            n_heads if n_heads is not None else src_heads, chunk_bytes, src_blocks,
                            dst_blocks, ready, max_ctas, status, span, threads)


def copy_segments(segs: torch.Tensor, total_bytes: int, ready: int = 0, max_ctas: int = 0,
                  status: Optional[torch.Tensor] = None) -> int:
    """Copy (src, dst, bytes) int64 segments (16-byte aligned) with SM loads/stores."""
    _n()
    return _C.copy_segments(segs, total_bytes, ready, max_ctas, status)


def wait_flag(flag_addr: int, target: int, status: torch.Tensor, timeout_s: float = 2.0) -> None:
    """Stream-ordered bounded wait until the u32 at ``flag_addr`` reaches ``target``."""
    _C.wait_flag(flag_addr, target & 0xFFFFFFFF, int(timeout_s * 1e9), status)
    _n()


def write_flag(flag_addr: int, value: int, like: torch.Tensor, add: bool = False) -> None:
    _C.write_flag(flag_addr, value & 0xFFFFFFFF, add, like)
    _n()


ipc_export = _C.ipc_export
ipc_open = _C.ipc_open
ipc_close = _C.ipc_close
enable_peer_access = _C.enable_peer_access
from_ptr = _C.from_ptr

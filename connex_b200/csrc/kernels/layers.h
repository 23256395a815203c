// Host entry points of the runtime kernels (layers.cu, attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdexcept>

namespace cx {

void rmsnorm(const void* x, int ldx, void* residual, int ldr, const void* w, void* out, int ldo, int T, int H,
             float eps, cudaStream_t s);
void rope_cache(void* qkv, int ldq, const int* pos, const float* cos_sin, const int64_t* slots, void* kc, void* vc,
                int T, int Hq, int Hkv, int D, int BS, int num_blocks, int max_pos, int* status, cudaStream_t s,
                const void* q_norm = nullptr, const void* k_norm = nullptr, float eps = 1e-6f);
void embedding(const int* ids, const void* table, void* out, int T, int H, int V, int* status, cudaStream_t s);
void argmax(const void* logits, int ldl, int B, int V, int* out, cudaStream_t s);
void gather_rows(const void* src, int lds, const int* idx, void* out, int ldo, int n, int H, cudaStream_t s);

// Causal varlen prefill attention (GQA, head_dim 128) on the tcgen05 tensor
// cores.  q/k/v rows live in the fused QKV buffer [T, (Hq+2Hkv)*128];
// tile_info: [n_tiles, 3] int32 of (seq start row, seq length, first query of
// the tile); tile_rows: 256 (two 128-row Q tiles per CTA) or 128 (one).
// qkv_cols = (Hq+2Hkv)*128, T = rows of qkv.
void prefill_attention_tc(const void* qkv, int ldq, int qkv_cols, int T, void* out, int ldo, const int* tile_info,
                          int n_tiles, int Hq, int Hkv, float scale, int* status, cudaStream_t s, int tile_rows);
// How many of every 8 softmax exponentials of the prefill attention run on
// the FMA pipe instead of the special-function unit: 0 (default), 2 or 4.
void attention_exp_split(int n);
// Device address of a zeroed u64 buffer [CTAs x 16] for the two-tile prefill
// attention's per-CTA cycle counters (0: off).
void attention_profile(int64_t ptr);

// The same over a paged cache (chunked prefill): q rows from QKV; K/V of the
// whole context from the caches [blocks, Hkv, 16, 128] (cache_rows =
// blocks * Hkv * 16) through block_tables [B, bt_stride]; tile_info: [n_tiles,
// 5] int32 of (seq start row, new tokens, first query, context length,
// sequence index).
void prefill_attention_paged_tc(const void* qkv, int ldq, int qkv_cols, int T, const void* kc, const void* vc,
                                int64_t cache_rows, const int* block_tables, int bt_stride, void* out, int ldo,
                                const int* tile_info, int n_tiles, int Hq, int Hkv, float scale, int* status,
                                cudaStream_t s, int tile_rows);

// Paged decode attention.  q: [B, *] rows (ld ldq, q heads first).
// Caches [blocks, Hkv, BS, 128]; block_tables [B, max_blocks]; ctx_lens [B].
// workspace: fp32, at least B*Hq*decode_attention_splits(max_ctx)*(128+2)
// floats; ws_floats >= 0 (its size) lets small batches use more splits.
void decode_attention(const void* q, int ldq, const void* kc, const void* vc, const int* block_tables,
                      int max_blocks, const int* ctx_lens, void* out, int ldo, int B, int Hq, int Hkv, int BS,
                      int max_ctx, float scale, float* workspace, cudaStream_t s, long ws_floats = -1,
                      int* status = nullptr, long cache_blocks = -1);
int decode_attention_splits(int max_ctx);
// Splits a launch uses (>= decode_attention_splits; more for small batches when ws_floats allows).
int decode_attention_plan(int B, int Hq, int Hkv, int max_ctx, long ws_floats);

}  // namespace cx

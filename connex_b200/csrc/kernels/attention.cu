// Paged decode attention of the serving runtime (head_dim 128, GQA).
//
// One query token per sequence against its paged KV cache ([blocks, Hkv, 16,
// 128] per layer, i.e. one head of one block is 4 KB contiguous).  Split-K
// over the context (512 tokens per CTA), one CTA per (sequence, kv head,
// split) computing all q heads of the GQA group, then a log-sum-exp merge of
// the splits.  (Prefill attention runs on tcgen05: attention_tc.cu.)
#include <algorithm>

#include "common.cuh"
#include "gemm.h"
#include "layers.h"

namespace cx {

// ------------------------------------------------------- paged decode
namespace dec {
constexpr int D = 128;
constexpr int SPLIT = 512;
constexpr int THREADS = 128;
constexpr int MAXG = 8;
}  // namespace dec

int decode_attention_splits(int max_ctx) { return (max_ctx + dec::SPLIT - 1) / dec::SPLIT; }

int decode_attention_plan(int B, int Hq, int Hkv, int max_ctx, long ws_floats) {
  int n = decode_attention_splits(max_ctx);
  if (ws_floats < 0 || B <= 0) return n;
  const long want = 2L * num_sms();
  if ((long)B * Hkv * n < want) {
    long n2 = (want + (long)B * Hkv - 1) / ((long)B * Hkv);
    n2 = std::min<long>(n2, (max_ctx + 63) / 64);
    n2 = std::min<long>(n2, ws_floats / ((long)B * Hq * (dec::D + 2)));
    if (n2 > n) n = (int)n2;
  }
  return n;
}

template <int G>
__global__ void __launch_bounds__(dec::THREADS)
    decode_attn_kernel(const __nv_bfloat16* __restrict__ q, int ldq, const __nv_bfloat16* __restrict__ kc,
                       const __nv_bfloat16* __restrict__ vc, const int* __restrict__ block_tables, int max_blocks,
                       const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out, int ldo, int Hq, int Hkv,
                       int BS, float scale_log2, float* __restrict__ ws, int n_splits, int split_len) {
  using namespace dec;
  const int b = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = ctx_lens[b];
  const int t0 = sp * split_len;
  const int t1 = min(ctx, t0 + split_len);  // split_len <= SPLIT: fits lg[][]
  const int n = t1 - t0;
  __shared__ float qs[G][D];
  __shared__ float lg[G][SPLIT];
  __shared__ float red[4][G][D];
  __shared__ float mls[G][2];
  const int* bt = block_tables + (size_t)b * max_blocks;

  if (n <= 0) {
    if (n_splits > 1 && tid < G) {
      float* ml = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)((g * G + tid) * n_splits + sp) * (D + 2);
      ml[D] = -INFINITY;
      ml[D + 1] = 0.f;
    }
    return;
  }
  for (int i = tid; i < G * D; i += THREADS) {
    const int h = i / D, d = i - h * D;
    qs[h][d] = __bfloat162float(q[(size_t)b * ldq + (size_t)(g * G + h) * D + d]) * scale_log2;
  }
  __syncthreads();
  // phase 1: logits.  4 threads per token; thread `sub` takes dims
  // v*32 + sub*8 + [0, 8) for v = 0..3, so the 4 threads of a token read q
  // from 4 different shared-memory banks (no conflicts; tokens broadcast).
  {
    const int sub = tid & 3;
    for (int base = 0; base < n; base += THREADS / 4) {
      const int tl = base + (tid >> 2);
      float acc[G];
#pragma unroll
      for (int h = 0; h < G; ++h) acc[h] = 0.f;
      if (tl < n) {
        const int t = t0 + tl;
        const int blk = bt[t / BS];
        const __nv_bfloat16* kr = kc + (((size_t)blk * Hkv + g) * BS + (t % BS)) * D + sub * 8;
        u128 kv4[4];
#pragma unroll
        for (int v = 0; v < 4; ++v) kv4[v] = ld_nc_v4(kr + v * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint32_t* pk = reinterpret_cast<const uint32_t*>(&kv4[v]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a = bf16_lo(pk[j]), c = bf16_hi(pk[j]);
            const int d = v * 32 + sub * 8 + 2 * j;
#pragma unroll
            for (int h = 0; h < G; ++h) acc[h] += a * qs[h][d] + c * qs[h][d + 1];
          }
        }
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
      }
      if (tl < n && sub == 0) {
#pragma unroll
        for (int h = 0; h < G; ++h) lg[h][tl] = acc[h];
      }
    }
  }
  __syncthreads();
  // phase 2: softmax statistics, one warp per head
  for (int h = warp; h < G; h += 4) {
    float mx = -INFINITY;
    for (int i = lane; i < n; i += 32) mx = fmaxf(mx, lg[h][i]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float p = exp2f(lg[h][i] - mx);
      lg[h][i] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      mls[h][0] = mx;
      mls[h][1] = sum;
    }
  }
  __syncthreads();
  // phase 3: P.V.  16 threads per token (8 dims each), 8 tokens in parallel.
  {
    const int dg = tid & 15, tp = tid >> 4;
    float acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;
    constexpr int VU = 4;  // V rows in flight per thread
    for (int tl0 = tp; tl0 < n; tl0 += 8 * VU) {
      u128 vv[VU];
#pragma unroll
      for (int u = 0; u < VU; ++u) {
        const int tl = tl0 + 8 * u;
        if (tl < n) {
          const int t = t0 + tl;
          const int blk = bt[t / BS];
          vv[u] = ld_nc_v4(vc + (((size_t)blk * Hkv + g) * BS + (t % BS)) * D + dg * 8);
        }
      }
#pragma unroll
      for (int u = 0; u < VU; ++u) {
        const int tl = tl0 + 8 * u;
        if (tl < n) {
          const uint32_t* pv = reinterpret_cast<const uint32_t*>(&vv[u]);
          float vf[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            vf[2 * j] = bf16_lo(pv[j]);
            vf[2 * j + 1] = bf16_hi(pv[j]);
          }
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float p = lg[h][tl];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[h][e] += p * vf[e];
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] += __shfl_xor_sync(0xffffffffu, acc[h][e], 16);
    if (lane < 16) {
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) red[warp][h][dg * 8 + e] = acc[h][e];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += THREADS) {
    const int h = i / D, d = i - h * D;
    const float v = red[0][h][d] + red[1][h][d] + red[2][h][d] + red[3][h][d];
    if (n_splits == 1) {
      out[(size_t)b * ldo + (size_t)(g * G + h) * D + d] = __float2bfloat16(v / mls[h][1]);
    } else {
      float* ml = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)((g * G + h) * n_splits + sp) * (D + 2);
      ml[d] = v;
      if (d == 0) {
        ml[D] = mls[h][0];
        ml[D + 1] = mls[h][1];
      }
    }
  }
}

__global__ void decode_merge_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int ldo, int Hq,
                                    int n_splits) {
  constexpr int D = dec::D;
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const float* base = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)h * n_splits * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, base[s * (D + 2) + D]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < n_splits; ++s) {
    const float m = base[s * (D + 2) + D];
    if (m == -INFINITY) continue;
    const float w = exp2f(m - M);
    num += base[s * (D + 2) + d] * w;
    den += base[s * (D + 2) + D + 1] * w;
  }
  out[(size_t)b * ldo + (size_t)h * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

void decode_attention(const void* q, int ldq, const void* kc, const void* vc, const int* block_tables,
                      int max_blocks, const int* ctx_lens, void* out, int ldo, int B, int Hq, int Hkv, int BS,
                      int max_ctx, float scale, float* workspace, cudaStream_t s, long ws_floats) {
  if (B == 0) return;
  const int G = Hq / Hkv;
  const int n_splits = decode_attention_plan(B, Hq, Hkv, max_ctx, ws_floats);
  const int split_len = (max_ctx + n_splits - 1) / n_splits;
  dim3 grid(B, Hkv, n_splits);
  auto Q = reinterpret_cast<const __nv_bfloat16*>(q);
  auto K = reinterpret_cast<const __nv_bfloat16*>(kc);
  auto V = reinterpret_cast<const __nv_bfloat16*>(vc);
  auto O = reinterpret_cast<__nv_bfloat16*>(out);
  const float sl = scale * 1.4426950408889634f;
  if (G == 4)
    decode_attn_kernel<4><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits, split_len);
  else if (G == 8)
    decode_attn_kernel<8><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits, split_len);
  else if (G == 1)
    decode_attn_kernel<1><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits, split_len);
  else if (G == 2)
    decode_attn_kernel<2><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits, split_len);
  else
    throw std::runtime_error("cx decode attention: GQA group size must be 1, 2, 4 or 8");
  if (n_splits > 1) decode_merge_kernel<<<dim3(B, Hq), dec::D, 0, s>>>(workspace, O, ldo, Hq, n_splits);
}

}  // namespace cx

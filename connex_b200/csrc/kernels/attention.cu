// Attention kernels of the serving runtime (head_dim 128, GQA).
//
// prefill_attention: causal attention over a packed batch of prompts whose
//   q/k/v rows sit in the fused QKV projection output.  Flash-attention
//   structure: one CTA per (64-query tile, q head), 4 warps x 16 query rows,
//   64-key tiles double-buffered in XOR-swizzled shared memory by cp.async,
//   online softmax in fp32 (exp2 domain), bf16 tensor-core MMAs
//   (mma.sync m16n8k16) for S = Q.K^T and O += P.V.
//
// decode_attention: one query token per sequence against its paged KV cache
//   ([blocks, Hkv, 16, 128] per layer, i.e. one head of one block is 4 KB
//   contiguous).  Split-K over the context (512 tokens per CTA), one CTA per
//   (sequence, kv head, split) computing all q heads of the GQA group, then a
//   log-sum-exp merge of the splits.
#include "common.cuh"
#include "layers.h"

namespace cx {

namespace fa {
constexpr int D = 128;
constexpr int BM = 64;
constexpr int BN = 64;
constexpr int THREADS = 128;
constexpr int TILE_BYTES = BM * D * 2;  // 16 KB
constexpr int SMEM = TILE_BYTES * 5;    // Q + 2x K + 2x V

// byte offset of 16-byte chunk `c` of row `r` in a [rows][128] bf16 tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Load `BM` rows x 128 dims starting at packed row `row0` (rows >= row_end are zero-filled).
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* base, int ld, int row0,
                                          int row_end) {
  for (int i = threadIdx.x; i < BM * 16; i += THREADS) {
    const int r = i >> 4, c = i & 15;
    const bool valid = row0 + r < row_end;
    const __nv_bfloat16* src = base + (size_t)(valid ? row0 + r : row0) * ld + c * 8;
    cp_async16(sbase + swz(r, c), src, valid);
  }
}
}  // namespace fa

__global__ void __launch_bounds__(fa::THREADS) prefill_attn_kernel(const __nv_bfloat16* __restrict__ qkv, int ldq,
                                                                    __nv_bfloat16* __restrict__ out, int ldo,
                                                                    const int* __restrict__ tile_info, int Hq,
                                                                    int Hkv, float scale_log2) {
  using namespace fa;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + TILE_BYTES, sV0 = sQ + 3 * TILE_BYTES;

  const int tile = blockIdx.x, h = blockIdx.y;
  const int seq_start = tile_info[tile * 3 + 0];
  const int seq_len = tile_info[tile * 3 + 1];
  const int q0 = tile_info[tile * 3 + 2];
  const int kvh = h / (Hq / Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const __nv_bfloat16* Qb = qkv + (size_t)h * D;
  const __nv_bfloat16* Kb = qkv + (size_t)(Hq + kvh) * D;
  const __nv_bfloat16* Vb = qkv + (size_t)(Hq + Hkv + kvh) * D;
  const int end = seq_start + seq_len;
  const int kv_len = min(seq_len, q0 + BM);
  const int nkv = (kv_len + BN - 1) / BN;

  load_tile(sQ, Qb, ldq, seq_start + q0, end);
  cp_async_commit();
  load_tile(sK0, Kb, ldq, seq_start, end);
  load_tile(sV0, Vb, ldq, seq_start, end);
  cp_async_commit();

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int qr0 = q0 + warp * 16 + (lane >> 2);  // query position (within seq) of c0/c1
  const int qr1 = qr0 + 8;                       // of c2/c3

  for (int j = 0; j < nkv; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkv) {
      const int nb = (j + 1) & 1;
      load_tile(sK0 + nb * TILE_BYTES, Kb, ldq, seq_start + (j + 1) * BN, end);
      load_tile(sV0 + nb * TILE_BYTES, Vb, ldq, seq_start + (j + 1) * BN, end);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(sQ + swz(r, c), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    const uint32_t sK = sK0 + buf * TILE_BYTES, sV = sV0 + buf * TILE_BYTES;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int nb2 = 0; nb2 < 4; ++nb2) {
        uint32_t k0, k1, k2, k3;
        const int r = nb2 * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(sK + swz(r, c), k0, k1, k2, k3);
        mma16816(s[nb2 * 2], qf[ks], k0, k1);
        mma16816(s[nb2 * 2 + 1], qf[ks], k2, k3);
      }
    }
    // scale + causal / length mask, row maxima
    float mx0 = m0, mx1 = m1;
    const bool need_mask = (j * BN + BN - 1 > q0 + warp * 16) || ((j + 1) * BN > seq_len);
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[nb][e] * scale_log2;
        if (need_mask) {
          const int key = j * BN + nb * 8 + 2 * (lane & 3) + (e & 1);
          const int qr = (e < 2) ? qr0 : qr1;
          if (key > qr || key >= seq_len) v = -INFINITY;
        }
        s[nb][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nb][0], s[nb][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nb][2], s[nb][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = (mx0 == -INFINITY) ? 1.f : exp2f(m0 - mx0);
    const float c1 = (mx1 == -INFINITY) ? 1.f : exp2f(m1 - mx1);
    const float b0 = (mx0 == -INFINITY) ? 0.f : mx0;
    const float b1 = (mx1 == -INFINITY) ? 0.f : mx1;
    m0 = mx0;
    m1 = mx1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      s[nb][0] = exp2f(s[nb][0] - b0);
      s[nb][1] = exp2f(s[nb][1] - b0);
      s[nb][2] = exp2f(s[nb][2] - b1);
      s[nb][3] = exp2f(s[nb][3] - b1);
      ps0 += s[nb][0] + s[nb][1];
      ps1 += s[nb][2] + s[nb][3];
    }
    l0 = l0 * c0 + ps0;
    l1 = l1 * c1 + ps1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= c0;
      o[i][1] *= c0;
      o[i][2] *= c1;
      o[i][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int db2 = 0; db2 < 8; ++db2) {
        uint32_t v0, v1, v2, v3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = db2 * 2 + (lane >> 4);
        ldsm_x4_t(sV + swz(r, c), v0, v1, v2, v3);
        mma16816(o[db2 * 2], pa, v0, v1);
        mma16816(o[db2 * 2 + 1], pa, v2, v3);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  __nv_bfloat16* ob = out + (size_t)h * D;
#pragma unroll
  for (int db = 0; db < 16; ++db) {
    const int col = db * 8 + 2 * (lane & 3);
    if (qr0 < seq_len)
      *reinterpret_cast<uint32_t*>(ob + (size_t)(seq_start + qr0) * ldo + col) =
          pack_bf16x2(o[db][0] * i0, o[db][1] * i0);
    if (qr1 < seq_len)
      *reinterpret_cast<uint32_t*>(ob + (size_t)(seq_start + qr1) * ldo + col) =
          pack_bf16x2(o[db][2] * i1, o[db][3] * i1);
  }
}

void prefill_attention(const void* qkv, int ldq, void* out, int ldo, const int* tile_info, int n_tiles, int Hq,
                       int Hkv, float scale, cudaStream_t s) {
  if (n_tiles == 0) return;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::SMEM);
    attr[dev & 63] = true;
  }
  dim3 grid(n_tiles, Hq);
  prefill_attn_kernel<<<grid, fa::THREADS, fa::SMEM, s>>>(reinterpret_cast<const __nv_bfloat16*>(qkv), ldq,
                                                           reinterpret_cast<__nv_bfloat16*>(out), ldo, tile_info, Hq,
                                                           Hkv, scale * 1.4426950408889634f);
}

// ------------------------------------------------------- paged decode
namespace dec {
constexpr int D = 128;
constexpr int SPLIT = 512;
constexpr int THREADS = 128;
constexpr int MAXG = 8;
}  // namespace dec

int decode_attention_splits(int max_ctx) { return (max_ctx + dec::SPLIT - 1) / dec::SPLIT; }

template <int G>
__global__ void __launch_bounds__(dec::THREADS)
    decode_attn_kernel(const __nv_bfloat16* __restrict__ q, int ldq, const __nv_bfloat16* __restrict__ kc,
                       const __nv_bfloat16* __restrict__ vc, const int* __restrict__ block_tables, int max_blocks,
                       const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out, int ldo, int Hq, int Hkv,
                       int BS, float scale_log2, float* __restrict__ ws, int n_splits) {
  using namespace dec;
  const int b = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = ctx_lens[b];
  const int t0 = sp * SPLIT;
  const int t1 = min(ctx, t0 + SPLIT);
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
  // phase 1: logits.  4 threads per token, 32 dims each.
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
        const __nv_bfloat16* kr = kc + (((size_t)blk * Hkv + g) * BS + (t % BS)) * D + sub * 32;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          u128 kv = ld_nc_v4(kr + v * 8);
          const uint32_t* pk = reinterpret_cast<const uint32_t*>(&kv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a = bf16_lo(pk[j]), c = bf16_hi(pk[j]);
            const int d = sub * 32 + v * 8 + 2 * j;
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
    for (int tl = tp; tl < n; tl += 8) {
      const int t = t0 + tl;
      const int blk = bt[t / BS];
      u128 vv = ld_nc_v4(vc + (((size_t)blk * Hkv + g) * BS + (t % BS)) * D + dg * 8);
      const uint32_t* pv = reinterpret_cast<const uint32_t*>(&vv);
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
                      int max_ctx, float scale, float* workspace, cudaStream_t s) {
  if (B == 0) return;
  const int G = Hq / Hkv;
  const int n_splits = decode_attention_splits(max_ctx);
  dim3 grid(B, Hkv, n_splits);
  auto Q = reinterpret_cast<const __nv_bfloat16*>(q);
  auto K = reinterpret_cast<const __nv_bfloat16*>(kc);
  auto V = reinterpret_cast<const __nv_bfloat16*>(vc);
  auto O = reinterpret_cast<__nv_bfloat16*>(out);
  const float sl = scale * 1.4426950408889634f;
  if (G == 4)
    decode_attn_kernel<4><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits);
  else if (G == 8)
    decode_attn_kernel<8><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits);
  else if (G == 1)
    decode_attn_kernel<1><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits);
  else if (G == 2)
    decode_attn_kernel<2><<<grid, dec::THREADS, 0, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo,
                                                         Hq, Hkv, BS, sl, workspace, n_splits);
  else
    throw std::runtime_error("cx decode attention: GQA group size must be 1, 2, 4 or 8");
  if (n_splits > 1) decode_merge_kernel<<<dim3(B, Hq), dec::D, 0, s>>>(workspace, O, ldo, Hq, n_splits);
}

}  // namespace cx

// Paged decode attention of the serving runtime (head_dim 128, GQA).
//
// One query token per sequence against its paged KV cache ([blocks, Hkv, 16,
// 128] per layer, i.e. one head of one block is 4 KB contiguous).  Split-K
// over the context (up to 512 tokens per CTA), one CTA per (sequence, kv
// head, split) computing all q heads of the GQA group, then a log-sum-exp
// merge of the splits.  (Prefill attention runs on tcgen05: attention_tc.cu.)
//
// The 16-token-block path is one pass per split: a producer warp streams the
// K and V head slices of two blocks per stage into a 3-stage shared-memory
// ring with bulk async copies (cp.async.bulk, 4 KB each, completing on an
// mbarrier; local memory only, no multicast), so a CTA keeps 48 KB of cache
// reads in flight with one thread; four consumer warps compute the stage's
// logits (q of the thread's dims held in registers), update the online
// softmax (one warp per head) and accumulate P.V, then release the stage.  Every wait is bounded and the consumers agree on
// a timeout with a barrier reduction, so none is left at a barrier.
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

// ------------------------------------------- pipelined path (16-token blocks)
namespace decb {
constexpr int D = 128, BS = 16, BPS = 2, TOK = BS * BPS, NS = 3;
constexpr int SLICE = BS * D * 2;            // one head of one block: 4 KB
constexpr int STAGE = 2 * BPS * SLICE;       // K and V of BPS blocks: 16 KB
constexpr int CONS = 128, THREADS = CONS + 32;
constexpr int MAXB = 64;                     // block ids of a split staged in shared memory (splits <= 1024 tokens)
template <int G>
constexpr int smem_bytes() {  // the token quarters' partial sums reuse the ring once it is drained
  return NS * STAGE + (G * D + 2 * G * TOK + 2 * 8 + 2 * 8 + MAXB) * 4 + 2 * NS * 8 + 16;
}
static_assert(3 * 8 * D * 4 <= NS * STAGE, "partial sums fit in the drained ring");
}  // namespace decb

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// every consumer thread's `ok`, AND-ed (a barrier of the 128 consumer threads)
__device__ __forceinline__ bool consumers_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

template <int G>
__global__ void __launch_bounds__(decb::THREADS, G >= 8 ? 2 : G >= 4 ? 3 : 4)
    decode_attn_bulk_kernel(const __nv_bfloat16* __restrict__ q, int ldq, const __nv_bfloat16* __restrict__ kc,
                            const __nv_bfloat16* __restrict__ vc, const int* __restrict__ block_tables,
                            int max_blocks, const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out,
                            int ldo, int Hq, int Hkv, float scale_log2, float* __restrict__ ws, int n_splits,
                            int split_len, int* status) {
  using namespace decb;
  extern __shared__ __align__(128) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem + NS * STAGE);  // [G][D], scaled to log2 units
  float* ps = qs + G * D;                                    // [2][G][TOK]: logits, then probabilities
  float* ml = ps + 2 * G * TOK;                              // [8] running max, [8] running sum
  float* al = ml + 16;                                       // [2][8] rescale factor of the stage
  float* part = reinterpret_cast<float*>(smem);             // [3][G][D]: quarters 1-3's sums, after the ring
  int* bids = reinterpret_cast<int*>(al + 16);               // [MAXB] the split's block ids
  uint64_t* full = reinterpret_cast<uint64_t*>(bids + MAXB);
  uint64_t* empty = full + NS;
  const int b = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = ctx_lens[b];
  const int t0 = sp * split_len;                             // split_len is a multiple of BS
  const int n = min(ctx, t0 + split_len) - t0;
  if (n <= 0) {
    if (n_splits > 1 && tid < G) {
      float* o = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)((g * G + tid) * n_splits + sp) * (D + 2);
      o[D] = -INFINITY;
      o[D + 1] = 0.f;
    }
    return;
  }
  const int nblk = (n + BS - 1) / BS, n_it = (nblk + BPS - 1) / BPS;
  const int* bt = block_tables + (size_t)b * max_blocks + t0 / BS;
  if (nblk > MAXB) {  // the host sizes splits so this never happens
    record_status(status, CX_ERR_BOUNDS);
    return;
  }
  // all block ids of the split in one parallel load: the producer then issues
  // its copies without a dependent global load in front of each
  for (int i = tid; i < nblk; i += THREADS) bids[i] = bt[i];
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONS);
    }
    fence_barrier_init();
  }
  for (int i = tid; i < G * D; i += THREADS) {
    const int h = i / D, d = i - h * D;
    qs[i] = __bfloat162float(q[(size_t)b * ldq + (size_t)(g * G + h) * D + d]) * scale_log2;
  }
  if (tid < 8) {
    ml[tid] = -INFINITY;
    ml[8 + tid] = 0.f;
  }
  __syncthreads();

  if (warp == CONS / 32) {  // producer
    if (lane == 0) {
      int it = 0;
      for (; it < n_it; ++it) {
        const int s = it % NS;
        if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, status)) break;
        const int nb = min(BPS, nblk - it * BPS);
        mbar_arrive_expect_tx(&full[s], (uint32_t)(nb * 2 * SLICE));
        uint8_t* stg = smem + s * STAGE;
        for (int bb = 0; bb < nb; ++bb) {
          const size_t off = ((size_t)bids[it * BPS + bb] * Hkv + g) * BS * D;
          bulk_load(stg + bb * SLICE, kc + off, SLICE, &full[s]);
          bulk_load(stg + (BPS + bb) * SLICE, vc + off, SLICE, &full[s]);
        }
      }
      // the CTA's shared memory must outlive every copy issued into it
      for (int j = max(0, it - NS); j < it; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, status);
    }
    return;
  }

  // consumers.  Logits: TPT = 2G threads per token, each owning DPT = 64 / G
  // dims of q for all G heads in registers (64 values whatever G is).  P.V:
  // thread (dim quad dq, token quarter qt) accumulates 4 dims of all G heads
  // over 8 tokens of each stage.
  // threads per token: 2G (measured: 16 threads for G = 4 fit four CTAs per
  // SM but their longer shuffle reductions cost the time the occupancy won)
  constexpr int TPT = 2 * G, DPT = D / TPT, NCH = DPT / 8, TPP = CONS / TPT;
  const int sub = tid % TPT, tk = tid / TPT;
  const int dq = tid & 31, qt = tid >> 5;
  uint64_t qr2[G][DPT / 2];  // q of the thread's dims, as packed pairs
  // the thread's dims: 16-byte chunks sub, sub + TPT, ... of the 256-byte row,
  // so the TPT threads of a token read one contiguous span per load
  // (conflict-free for G >= 4) and every q register is indexed statically
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int j = 0; j < NCH; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float* qp = qs + h * D + (sub + j * TPT) * 8 + 2 * e;
        qr2[h][j * 4 + e] = f32x2(qp[0], qp[1]);
      }
  uint64_t acc[G][2];  // dims (4dq, 4dq+1) and (4dq+2, 4dq+3) of each head, packed
#pragma unroll
  for (int h = 0; h < G; ++h) acc[h][0] = acc[h][1] = 0ull;
  bool ok = true;
  for (int it = 0; it < n_it; ++it) {
    const int s = it % NS;
    ok = consumers_all(mbar_wait(&full[s], (it / NS) & 1, status));
    if (!ok) break;
    const uint8_t* stg = smem + s * STAGE;
    float* pb = ps + (it & 1) * G * TOK;
    float* ab = al + (it & 1) * 8;
#pragma unroll
    for (int pass = 0; pass * TPP < TOK; ++pass) {
      const int tt = pass * TPP + tk;
      float a[G];
      if (tt < TOK) {
        // two dims per packed f32x2 FMA: (k0, k1) x (q0, q1) + (s0, s1), the lanes summed at the end
        uint64_t a2[G];
#pragma unroll
        for (int h = 0; h < G; ++h) a2[h] = 0ull;
        const uint8_t* krow = stg + (tt / BS) * SLICE + (tt % BS) * (D * 2);
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          const u128 kv = *reinterpret_cast<const u128*>(krow + (sub + j * TPT) * 16);
          const uint32_t* pk = reinterpret_cast<const uint32_t*>(&kv);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint64_t k2 = f32x2(bf16_lo(pk[w]), bf16_hi(pk[w]));
#pragma unroll
            for (int h = 0; h < G; ++h) a2[h] = fma_f32x2(k2, qr2[h][j * 4 + w], a2[h]);
          }
        }
#pragma unroll
        for (int h = 0; h < G; ++h) a[h] = lo_f32(a2[h]) + hi_f32(a2[h]);
      } else {
#pragma unroll
        for (int h = 0; h < G; ++h) a[h] = 0.f;
      }
#pragma unroll
      for (int off = 1; off < TPT; off <<= 1)
#pragma unroll
        for (int h = 0; h < G; ++h) a[h] += __shfl_xor_sync(0xffffffffu, a[h], off);
      if (sub == 0 && tt < TOK) {
        const int tok = it * TOK + tt;
#pragma unroll
        for (int h = 0; h < G; ++h) pb[h * TOK + tt] = tok < n ? a[h] : -INFINITY;
      }
    }
    consumers_sync();
    for (int h = warp; h < G; h += 4) {  // online softmax, one warp per head, one lane per token
      const float x = pb[h * TOK + lane];
      const float mx = warp_max(x);
      const float m_old = ml[h], m_new = fmaxf(m_old, mx);
      const float p = x == -INFINITY ? 0.f : exp2f(x - m_new);
      const float sum = warp_sum(p);
      const float alpha = m_old == -INFINITY ? 0.f : exp2f(m_old - m_new);
      pb[h * TOK + lane] = p;
      __syncwarp();
      if (lane == 0) {
        ml[h] = m_new;
        ml[8 + h] = ml[8 + h] * alpha + sum;
        ab[h] = alpha;
      }
    }
    consumers_sync();
    {  // P.V over this thread's quarter of the stage (8 tokens, 4 dims, all heads)
      const int base = it * TOK + qt * 8;
      const int cnt = min(8, n - base);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const uint64_t a2 = f32x2(ab[h], ab[h]);
        acc[h][0] = mul_f32x2(acc[h][0], a2);
        acc[h][1] = mul_f32x2(acc[h][1], a2);
      }
#pragma unroll
      for (int j4 = 0; j4 < 8; j4 += 4) {  // four tokens at a time: one float4 of p per head
        if (j4 < cnt) {
          float pr[G][4];
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float4 p4 = *reinterpret_cast<const float4*>(pb + h * TOK + qt * 8 + j4);
            pr[h][0] = p4.x; pr[h][1] = p4.y; pr[h][2] = p4.z; pr[h][3] = p4.w;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (j4 + j < cnt) {  // past the end: p is 0, but the slot's V may be NaN
              const int t = qt * 8 + j4 + j;
              const uint2 v4 = *reinterpret_cast<const uint2*>(stg + (BPS + t / BS) * SLICE + (t % BS) * (D * 2) +
                                                               dq * 8);
              const uint64_t v01 = f32x2(bf16_lo(v4.x), bf16_hi(v4.x)), v23 = f32x2(bf16_lo(v4.y), bf16_hi(v4.y));
#pragma unroll
              for (int h = 0; h < G; ++h) {
                const uint64_t pp = f32x2(pr[h][j], pr[h][j]);
                acc[h][0] = fma_f32x2(pp, v01, acc[h][0]);
                acc[h][1] = fma_f32x2(pp, v23, acc[h][1]);
              }
            }
          }
        }
      }
    }
    mbar_arrive(&empty[s]);
  }
  if (!ok) return;
  consumers_sync();  // every stage is consumed: the ring is free for the partial sums
  // quarters 1-3 hand their sums to quarter 0 through shared memory
  if (qt > 0) {
#pragma unroll
    for (int h = 0; h < G; ++h)
      *reinterpret_cast<float4*>(part + ((qt - 1) * G + h) * D + 4 * dq) =
          make_float4(lo_f32(acc[h][0]), hi_f32(acc[h][0]), lo_f32(acc[h][1]), hi_f32(acc[h][1]));
  }
  consumers_sync();
  if (qt == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float o[4] = {lo_f32(acc[h][0]), hi_f32(acc[h][0]), lo_f32(acc[h][1]), hi_f32(acc[h][1])};
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const float4 x = *reinterpret_cast<const float4*>(part + (k * G + h) * D + 4 * dq);
        o[0] += x.x; o[1] += x.y; o[2] += x.z; o[3] += x.w;
      }
      if (n_splits == 1) {
        const float inv = 1.f / ml[8 + h];
        uint2 w;
        w.x = pack_bf16x2(o[0] * inv, o[1] * inv);
        w.y = pack_bf16x2(o[2] * inv, o[3] * inv);
        *reinterpret_cast<uint2*>(out + (size_t)b * ldo + (size_t)(g * G + h) * D + 4 * dq) = w;
      } else {
        float* op = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)((g * G + h) * n_splits + sp) * (D + 2);
#pragma unroll
        for (int e = 0; e < 4; ++e) op[4 * dq + e] = o[e];
        if (dq == 0) {
          op[D] = ml[h];
          op[D + 1] = ml[8 + h];
        }
      }
    }
  }
}

// ------------------------------------- tensor-core path (16-token blocks)
// QK^T and P.V on mma.sync (bf16 in, fp32 accumulate): the kernel is memory
// bound, so the point is the instruction count -- a warp's logits for 8
// tokens x 128 dims are 8 MMAs instead of ~600 CUDA-core instructions.  K and
// V stream in by TMA (128-byte swizzle: the ldmatrix reads are conflict-free)
// into a 3-stage ring; warp w takes tokens [8w, 8w + 8) of every 32-token
// stage with its own online softmax (no barrier per stage) and the warps
// merge at the end.  S^T = q.K^T puts the heads on the M dimension (rows
// 0..7; rows 8..15 are zero padding); its C fragment (head, token pair) is
// exactly the B fragment of O^T = V^T.P^T (m16n8k8: dims on M, heads on N),
// so P never leaves the registers and O needs no padded rows.
namespace decm {
constexpr int D = 128, BS = 16, TOK = 32, NS = 3, SLICE = BS * D * 2, STAGE = 4 * SLICE;  // K0 K1 V0 V1
constexpr int CONS = 128, THREADS = CONS + 32, MAXB = 64;
// ring (1 KB aligned for the swizzle) | q [8][D] fp32 | per-warp (m, l) [4][8][2] | block ids | barriers
constexpr int SMEM = 1024 + NS * STAGE + 8 * D * 4 + 4 * 8 * 2 * 4 + MAXB * 4 + 2 * NS * 8;
}  // namespace decm

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D (16x8 fp32) += A (16x16 bf16, rows 8..15 zero) . B (16x8 bf16)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  const uint32_t z = 0u;
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(z), "r"(a2), "r"(z), "r"(b0), "r"(b1));
}
// D (16x8 fp32) += A (16x8 bf16) . B (8x8 bf16)
__device__ __forceinline__ void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
               "{%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(b0));
}

template <int G>
__global__ void __launch_bounds__(decm::THREADS, 3)
    decode_attn_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                           const __nv_bfloat16* __restrict__ q, int ldq, const int* __restrict__ block_tables,
                           int max_blocks, const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out, int ldo,
                           int Hq, int Hkv, float scale_log2, float* __restrict__ ws, int n_splits, int split_len,
                           int* status) {
  using namespace decm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* qs = reinterpret_cast<float*>(ring + NS * STAGE);  // [8][D]
  float* mlw = qs + 8 * D;                                  // [4 warps][8 heads][m, l]
  int* bids = reinterpret_cast<int*>(mlw + 4 * 8 * 2);
  uint64_t* full = reinterpret_cast<uint64_t*>(bids + MAXB);
  uint64_t* empty = full + NS;
  const int b = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = ctx_lens[b];
  const int t0 = sp * split_len;
  const int n = min(ctx, t0 + split_len) - t0;
  if (n <= 0) {
    if (n_splits > 1 && tid < G) {
      float* o = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)((g * G + tid) * n_splits + sp) * (D + 2);
      o[D] = -INFINITY;
      o[D + 1] = 0.f;
    }
    return;
  }
  const int nblk = (n + BS - 1) / BS, n_it = (nblk + 1) / 2;
  if (nblk > MAXB) {
    record_status(status, CX_ERR_BOUNDS);
    return;
  }
  const int* bt = block_tables + (size_t)b * max_blocks + t0 / BS;
  for (int i = tid; i < nblk; i += THREADS) bids[i] = bt[i];
  for (int i = tid; i < 8 * D; i += THREADS) {
    const int h = i / D, d = i - h * D;
    qs[i] = h < G ? __bfloat162float(q[(size_t)b * ldq + (size_t)(g * G + h) * D + d]) * scale_log2 : 0.f;
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONS / 32);
    }
    fence_barrier_init();
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  __syncthreads();

  if (warp == CONS / 32) {  // producer: TMA of two blocks' K and V head slices per stage
    if (lane == 0) {
      int it = 0;
      for (; it < n_it; ++it) {
        const int s = it % NS;
        if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, status)) break;
        const int nb = min(2, nblk - it * 2);
        mbar_arrive_expect_tx(&full[s], (uint32_t)(nb * 2 * SLICE));
        uint8_t* stg = ring + s * STAGE;
        for (int bb = 0; bb < nb; ++bb) {
          const int row = (bids[it * 2 + bb] * Hkv + g) * BS;  // cache row of (block, head, token 0)
          for (int h = 0; h < 2; ++h) {
            tma_load_2d(stg + bb * SLICE + h * 2048, &tmk, &full[s], h * 64, row);
            tma_load_2d(stg + (2 + bb) * SLICE + h * 2048, &tmv, &full[s], h * 64, row);
          }
        }
      }
      for (int j = max(0, it - NS); j < it; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, status);
    }
    return;
  }

  const int gq = lane >> 2, qd = lane & 3;  // fragment row (head) / column pair
  // q as the A operand of S^T = q.K^T: 8 k-steps of 16 dims, rows 0..7
  uint32_t qa[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const float* qp = qs + gq * D + kk * 16 + 2 * qd;
    qa[kk][0] = pack_bf16x2(qp[0], qp[1]);
    qa[kk][1] = pack_bf16x2(qp[8], qp[9]);
  }
  float o[8][4];  // O^T: m-tile mt = dims [16 mt, 16 mt + 16); (dim gq | gq + 8, heads 2qd, 2qd + 1)
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // row gq's running max / this thread's partial sum
  const int blk = warp >> 1, rib0 = (warp & 1) * 8;  // this warp's 8 tokens: rows rib0.. of block blk
  const int lrow = rib0 + (lane & 7), lmat = lane >> 3;  // ldmatrix: the row this lane addresses
  bool ok = true;
  for (int it = 0; it < n_it; ++it) {
    const int s = it % NS;
    if (!mbar_wait(&full[s], (it / NS) & 1, status)) { ok = false; break; }
    const uint8_t* stg = ring + s * STAGE;
    const int tok0 = it * TOK + warp * 8;  // first of this warp's tokens in the split
    if (tok0 < n) {
      const uint32_t kb = smem_u32(stg + blk * SLICE), vb = smem_u32(stg + (2 + blk) * SLICE);
      if (tok0 + 8 > n) {  // past the end: V rows are cache slots nobody wrote (NaN would survive P = 0)
        for (int i = lane; i < 8 * 16; i += 32) {
          const int r = i >> 4, c = i & 15;
          if (tok0 + r >= n)
            *reinterpret_cast<uint4*>(const_cast<uint8_t*>(stg) + (2 + blk) * SLICE + (c >> 3) * 2048 +
                                      (rib0 + r) * 128 + (((c & 7) ^ ((rib0 + r) & 7)) << 4)) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      float sc[4] = {0.f, 0.f, 0.f, 0.f};  // S^T: (head gq, tokens 2qd, 2qd + 1); rows 8.. unused
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {  // one ldmatrix.x4 = two k-steps of K^T
        const int chunk = kk * 2 + lmat;   // 16-byte chunk of the row: dims [8 chunk, 8 chunk + 8)
        const uint32_t addr = kb + (chunk >> 3) * 2048 + lrow * 128 + (((chunk & 7) ^ (lrow & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma16816(sc, qa[kk][0], qa[kk][1], b0, b1);
        mma16816(sc, qa[kk + 1][0], qa[kk + 1][1], b2, b3);
      }
      const float s0 = tok0 + 2 * qd < n ? sc[0] : -INFINITY;
      const float s1 = tok0 + 2 * qd + 1 < n ? sc[1] : -INFINITY;
      float mx = fmaxf(s0, s1);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
      const float p0 = s0 == -INFINITY ? 0.f : exp2f(s0 - m_new), p1 = s1 == -INFINITY ? 0.f : exp2f(s1 - m_new);
      l_run = l_run * alpha + p0 + p1;
      m_run = m_new;
      const uint32_t pb = pack_bf16x2(p0, p1);  // B fragment of P^T: (tokens 2qd, 2qd + 1; head gq)
      // O^T's columns are heads 2qd, 2qd + 1: their rescale factors live in rows 2qd, 2qd + 1
      const float a_lo = __shfl_sync(0xffffffffu, alpha, 8 * qd), a_hi = __shfl_sync(0xffffffffu, alpha, 8 * qd + 4);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= a_lo;
        o[mt][1] *= a_hi;
        o[mt][2] *= a_lo;
        o[mt][3] *= a_hi;
      }
#pragma unroll
      for (int mt = 0; mt < 8; mt += 2) {  // one ldmatrix.x4.trans = V^T of 32 dims (two m-tiles)
        const int chunk = 2 * mt + lmat;   // dims [8 chunk, 8 chunk + 8)
        const uint32_t addr = vb + (chunk >> 3) * 2048 + lrow * 128 + (((chunk & 7) ^ (lrow & 7)) << 4);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(addr, v0, v1, v2, v3);
        mma1688(o[mt], v0, v1, pb);
        mma1688(o[mt + 1], v2, v3, pb);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  ok = consumers_all(ok);
  if (!ok) return;
  // merge the four warps: (m, l) per head, then the weighted sums of O
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (qd == 0) {
    mlw[(warp * 8 + gq) * 2] = m_run;
    mlw[(warp * 8 + gq) * 2 + 1] = l_run;
  }
  consumers_sync();  // the ring is drained: reuse it for the warps' O
  float* ow = reinterpret_cast<float*>(ring);  // [4 warps][8 heads][D]
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d0 = mt * 16 + gq;
    ow[(warp * 8 + 2 * qd) * D + d0] = o[mt][0];
    ow[(warp * 8 + 2 * qd + 1) * D + d0] = o[mt][1];
    ow[(warp * 8 + 2 * qd) * D + d0 + 8] = o[mt][2];
    ow[(warp * 8 + 2 * qd + 1) * D + d0 + 8] = o[mt][3];
  }
  consumers_sync();
  for (int i = tid; i < G * D; i += CONS) {
    const int h = i / D, d = i - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mlw[(w * 8 + h) * 2]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = mlw[(w * 8 + h) * 2];
      if (mw == -INFINITY) continue;
      const float f = exp2f(mw - M);
      num += ow[(w * 8 + h) * D + d] * f;
      den += mlw[(w * 8 + h) * 2 + 1] * f;
    }
    if (n_splits == 1) {
      out[(size_t)b * ldo + (size_t)(g * G + h) * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
    } else {
      float* op = ws + (size_t)b * Hq * n_splits * (D + 2) + (size_t)((g * G + h) * n_splits + sp) * (D + 2);
      op[d] = num;
      if (d == 0) {
        op[D] = M;
        op[D + 1] = den;
      }
    }
  }
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
                      int max_ctx, float scale, float* workspace, cudaStream_t s, long ws_floats, int* status,
                      long cache_blocks) {
  if (B == 0) return;
  const int G = Hq / Hkv;
  const int n_splits = decode_attention_plan(B, Hq, Hkv, max_ctx, ws_floats);
  dim3 grid(B, Hkv, n_splits);
  auto Q = reinterpret_cast<const __nv_bfloat16*>(q);
  auto K = reinterpret_cast<const __nv_bfloat16*>(kc);
  auto V = reinterpret_cast<const __nv_bfloat16*>(vc);
  auto O = reinterpret_cast<__nv_bfloat16*>(out);
  const float sl = scale * 1.4426950408889634f;
  if (BS == decm::BS && (G == 1 || G == 2 || G == 4 || G == 8)) {
    const int split_len = ((max_ctx + n_splits - 1) / n_splits + decm::BS - 1) / decm::BS * decm::BS;
    const uint64_t rows = cache_blocks > 0 ? (uint64_t)cache_blocks * Hkv * decm::BS : (1ull << 31);
    const CUtensorMap tk = make_tmap_bf16_2d(kc, decm::D, rows, decm::D * 2, 64, 16, true);
    const CUtensorMap tv = make_tmap_bf16_2d(vc, decm::D, rows, decm::D * 2, 64, 16, true);
    auto launch = [&](auto kern) {
      static bool attr[64][4] = {};
      int dev;
      cudaGetDevice(&dev);
      const int gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
      if (!attr[dev & 63][gi]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, decm::SMEM);
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        attr[dev & 63][gi] = true;
      }
      kern<<<grid, decm::THREADS, decm::SMEM, s>>>(tk, tv, Q, ldq, block_tables, max_blocks, ctx_lens, O, ldo, Hq,
                                                    Hkv, sl, workspace, n_splits, split_len, status);
    };
    if (G == 4) launch(decode_attn_mma_kernel<4>);
    else if (G == 8) launch(decode_attn_mma_kernel<8>);
    else if (G == 2) launch(decode_attn_mma_kernel<2>);
    else launch(decode_attn_mma_kernel<1>);
    if (n_splits > 1) decode_merge_kernel<<<dim3(B, Hq), dec::D, 0, s>>>(workspace, O, ldo, Hq, n_splits);
    return;
  }
  if (BS == decb::BS && (G == 1 || G == 2 || G == 4 || G == 8)) {
    // splits start on block boundaries; n_splits * split_len still covers max_ctx
    const int split_len = ((max_ctx + n_splits - 1) / n_splits + decb::BS - 1) / decb::BS * decb::BS;
    auto launch = [&](auto kern, int smem) {
      static bool attr[64][4] = {};
      int dev;
      cudaGetDevice(&dev);
      const int gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
      if (!attr[dev & 63][gi]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);   // 4 CTAs per SM
        attr[dev & 63][gi] = true;
      }
      kern<<<grid, decb::THREADS, smem, s>>>(Q, ldq, K, V, block_tables, max_blocks, ctx_lens, O, ldo, Hq, Hkv, sl,
                                             workspace, n_splits, split_len, status);
    };
    if (G == 4) launch(decode_attn_bulk_kernel<4>, decb::smem_bytes<4>());
    else if (G == 8) launch(decode_attn_bulk_kernel<8>, decb::smem_bytes<8>());
    else if (G == 2) launch(decode_attn_bulk_kernel<2>, decb::smem_bytes<2>());
    else launch(decode_attn_bulk_kernel<1>, decb::smem_bytes<1>());
    if (n_splits > 1) decode_merge_kernel<<<dim3(B, Hq), dec::D, 0, s>>>(workspace, O, ldo, Hq, n_splits);
    return;
  }
  const int split_len = (max_ctx + n_splits - 1) / n_splits;
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

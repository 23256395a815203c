// Causal varlen prefill attention on the sm_100a tensor cores (tcgen05 + TMA + TMEM).
//
// One CTA per (128-query tile, q head); two CTAs per SM (112 KB shared
// memory and 256 TMEM columns each), so one CTA's softmax overlaps the other
// CTA's MMAs.  6 warps per CTA:
//   warp 0    : TMA producer.  Q once ([128 rows x 128 dims] as two 64-dim
//               boxes), then K and V of each 64-key tile into a 2-stage ring,
//               straight from the fused QKV buffer.
//   warp 1    : allocates TMEM (S0 | S1 | O = 64 + 64 + 128 columns); one
//               thread issues S_j = Q.K_j^T (M=128, N=64, K=128, both
//               K-major) into S[j%2] and O += P_{j-1}.V_{j-1} (A = P from
//               shared memory, B = V MN-major, N=128, K=64), so Q.K of the
//               next tile overlaps the current softmax.
//   warps 2-5 : softmax, one thread per query row (its TMEM lane): the 64
//               scores of the row are loaded once into registers, masked,
//               exponentiated (ex2.approx) and packed to bf16 before waiting
//               for the previous P.V; O in TMEM is rescaled lazily (only
//               when the running max grew by more than 2^8); P is written
//               into the 128-byte-swizzled K-major layout the MMA reads.
// All waits are bounded (status word on timeout); no cluster multicast.
//
// Paged variant (chunked prefill): the chunk's queries come from the QKV
// buffer, while K and V of the whole context -- earlier chunks and this
// one, already written by rope_cache -- stream from the paged cache through
// the sequence's block table: each 64-key tile is four 16-token blocks, each
// loaded as [16 rows x 64 dims] boxes into the same swizzled tile layout
// (a box lands at a 2 KB offset, so the 1 KB swizzle pattern is unchanged).
// Query i of a chunk with context c sits at position c + i and sees keys
// [0, c + i].
#include "common.cuh"
#include "gemm.h"
#include "layers.h"

namespace cx {

namespace fatc {
constexpr int D = 128;
constexpr int BM = 128;
constexpr int BN = 64;
constexpr int THREADS = 192;
constexpr int Q_HALF = 128 * 64 * 2;   // [128 rows x 64 dims]: 16 KB
constexpr int KV_HALF = 64 * 64 * 2;   // [64 rows x 64 dims]: 8 KB
constexpr int KV_TILE = 2 * KV_HALF;   // [64 keys x 128 dims]: 16 KB
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * Q_HALF;     // 2 stages
constexpr int OFF_V = OFF_K + 2 * KV_TILE;    // 2 stages
constexpr int OFF_P = OFF_V + 2 * KV_TILE;    // [128 q x 64 keys]: 16 KB
constexpr int OFF_BAR = OFF_P + 128 * 64 * 2;
constexpr int SMEM = OFF_BAR + 256;
constexpr int TMEM_COLS = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x of a pair on the FMA and integer pipes only (no special-function or
// conversion instruction), to take part of the softmax's exponentials off
// the special-function unit.  x = n + f with n = round(x) and f in
// [-0.5, 0.5]: adding 1.5 * 2^23 rounds x to an integer held in the low
// mantissa bits of the sum, so n is read from those bits and f = x - n is
// exact; 2^f comes from a cubic fitted here to 2^f on [-0.5, 0.5] as the
// minimax of the relative error (linear program over 4001 points; 7.5e-5 in
// fp32 Horner form, far below the bf16 rounding of P), and n is added to its
// exponent field.  Inputs are clamped to >= -125 (the result stays a normal
// float; 2^-125 next to the row's largest term, >= 2^-8, is as good as 0),
// which also maps the mask's -inf to that value.
constexpr float EXP2_C0 = 0.999928057f, EXP2_C1 = 0.693260968f, EXP2_C2 = 0.242611125f, EXP2_C3 = 0.0551716685f;
__device__ __forceinline__ uint64_t poly_exp2_x2(uint64_t x2) {
  const uint64_t x = f32x2(fmaxf(lo_f32(x2), -125.0f), fmaxf(hi_f32(x2), -125.0f));
  const uint64_t t = add_f32x2(x, f32x2(12582912.0f, 12582912.0f));
  const uint64_t n = add_f32x2(t, f32x2(-12582912.0f, -12582912.0f));
  const uint64_t f = fma_f32x2(n, f32x2(-1.0f, -1.0f), x);
  uint64_t p = fma_f32x2(f32x2(EXP2_C3, EXP2_C3), f, f32x2(EXP2_C2, EXP2_C2));
  p = fma_f32x2(p, f, f32x2(EXP2_C1, EXP2_C1));
  p = fma_f32x2(p, f, f32x2(EXP2_C0, EXP2_C0));
  const uint32_t lo = __float_as_uint(lo_f32(p)) + (__float_as_uint(lo_f32(t)) << 23);
  const uint32_t hi = __float_as_uint(hi_f32(p)) + (__float_as_uint(hi_f32(t)) << 23);
  return f32x2(__uint_as_float(lo), __uint_as_float(hi));
}
// 2^x of a bf16 pair with one packed special-function instruction.
__device__ __forceinline__ uint32_t exp2_bf16x2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// pair P of a row (elements 2P, 2P+1): EMU of every 8 elements (EMU / 2 of
// every 4 pairs) go to the polynomial, the rest to ex2.approx.  EMU is a
// template parameter of the kernel, chosen by attention_exp_split.
template <int EMU, int P>
__device__ __forceinline__ uint64_t exp2_pair(uint64_t t2) {
  if constexpr ((P % 4) >= 4 - EMU / 2) {
    return poly_exp2_x2(t2);
  } else {
    return f32x2(fast_exp2(lo_f32(t2)), fast_exp2(hi_f32(t2)));
  }
}


// MN-major, 128-byte-swizzled operand (V as the B operand of P.V): 64
// contiguous elements per 128-byte row (rows = K index), 8-row groups 1024 B
// apart (SBO), 64-element MN blocks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}
}  // namespace fatc

template <bool PAGED, int EMU>
__global__ void __launch_bounds__(fatc::THREADS, 2)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv, __nv_bfloat16* __restrict__ out, int ldo,
                           const int* __restrict__ tile_info, int n_tiles, int Hq, int Hkv, float scale_log2,
                           const int* __restrict__ block_tables, int bt_stride, int* status,
                           unsigned long long* /*prof: two-tile kernel only*/) {
  using namespace fatc;
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0) {  // swizzled operands need a 1 KB-aligned base
    if (threadIdx.x == 0) record_status(status, CX_ERR_BOUNDS);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]  K and V have their own rings: K_j is released as
  uint64_t* k_empty = bars + 3;   // [2]  soon as S_j = Q.K_j^T is done, so K_{j+2} streams in
  uint64_t* s_full = bars + 5;    // [2]  while softmax j / P_j.V_j are still running
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint64_t* v_full = bars + 12;   // [2]
  uint64_t* v_empty = bars + 14;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int tile = (int)blockIdx.x;  // tile_info lists the heaviest tiles first
  const int h = blockIdx.y;
  const int* ti = tile_info + tile * (PAGED ? 5 : 3);
  const int seq_start = ti[0];                    // first row of the sequence's new tokens in QKV
  const int seq_len = ti[1];                      // its new tokens
  const int q0 = ti[2];                           // first query of this tile (among the new tokens)
  const int ctx = PAGED ? ti[3] : 0;              // tokens already in the cache before them
  const int* bt = PAGED ? block_tables + (size_t)ti[4] * bt_stride : nullptr;
  const int total = ctx + seq_len;
  const int g = h / (Hq / Hkv);
  const int kv_len = min(total, ctx + q0 + BM);
  const int nkv = (kv_len + BN - 1) / BN;
  const int qcol = h * D, kcol = (Hq + g) * D, vcol = (Hq + Hkv + g) * D;

  const int warp = warp_id(), lane = lane_id();
  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    if (PAGED) prefetch_tmap(&tmv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS0 = tmem, tS1 = tmem + BN, tO = tmem + 2 * BN;

  if (warp == 0) {
    if (lane == 0) {
      const int row0 = seq_start + q0;
      mbar_arrive_expect_tx(q_full, 2 * Q_HALF);
      tma_load_2d(smem + OFF_Q, &tmq, q_full, qcol, row0);
      tma_load_2d(smem + OFF_Q + Q_HALF, &tmq, q_full, qcol + 64, row0);
      // paged: cache rows of the four 16-token blocks of a key tile (tile j's
      // block ids are fetched one tile ahead so their loads are in flight)
      constexpr int BPT = BN / 16;
      const int nblk = (total + 15) / 16;
      auto rows_of = [&](int j, int (&r)[BPT]) {
#pragma unroll
        for (int i = 0; i < BPT; ++i) {
          const int b = j * BPT + i;
          r[i] = (bt[b < nblk ? b : 0] * Hkv + g) * 16;  // past the end: any valid block (masked)
        }
      };
      auto load_tile = [&](const CUtensorMap* map, uint8_t* buf, uint64_t* bar, int col, int j, const int (&r)[BPT]) {
        if constexpr (PAGED) {
#pragma unroll
          for (int i = 0; i < BPT; ++i) {
            tma_load_2d(buf + i * 2048, map, bar, 0, r[i]);
            tma_load_2d(buf + KV_HALF + i * 2048, map, bar, 64, r[i]);
          }
        } else {
          tma_load_2d(buf, map, bar, col, seq_start + j * BN);
          tma_load_2d(buf + KV_HALF, map, bar, col + 64, seq_start + j * BN);
        }
      };
      int r_cur[BPT] = {}, r_prev[BPT] = {}, r_next[BPT] = {};
      if (PAGED) rows_of(0, r_cur);
      // K_j goes out before V_{j-1}: K stages free up earlier (after Q.K^T)
      auto load_k = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1, status)) return false;
        mbar_arrive_expect_tx(&k_full[s], KV_TILE);
        load_tile(&tmk, smem + OFF_K + s * KV_TILE, &k_full[s], kcol, j, r_cur);
        return true;
      };
      auto load_v = [&](int j, const int (&r)[BPT]) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&v_empty[s], ((j >> 1) & 1) ^ 1, status)) return false;
        mbar_arrive_expect_tx(&v_full[s], KV_TILE);
        load_tile(&tmv, smem + OFF_V + s * KV_TILE, &v_full[s], vcol, j, r);
        return true;
      };
      bool good = true;
      for (int j = 0; j < nkv && good; ++j) {
        good = load_k(j);
        if (PAGED && j + 1 < nkv) rows_of(j + 1, r_next);
        if (good && j >= 1) good = load_v(j - 1, r_prev);
#pragma unroll
        for (int i = 0; i < BPT; ++i) {
          r_prev[i] = r_cur[i];
          r_cur[i] = r_next[i];
        }
      }
      if (good) load_v(nkv - 1, r_prev);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = umma_idesc_bf16(BM, BN);
      constexpr uint32_t IDESC_PV = umma_idesc_bf16_bmn(BM, D);
      const uint32_t sQ = smem_u32(smem + OFF_Q), sP = smem_u32(smem + OFF_P);
      bool ok = mbar_wait(q_full, 0, status);
      bool issued = false;
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait(&v_full[jj & 1], (jj >> 1) & 1, status)) return false;
        if (!mbar_wait(p_full, jj & 1, status)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + OFF_V + (jj & 1) * KV_TILE);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          umma_bf16(tO, umma_desc_sw128(sP + kk * 32), umma_desc_sw128_mn(sV + kk * 2048, KV_HALF), IDESC_PV,
                    (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[jj & 1]);
        return true;
      };
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, status)) { ok = false; break; }
        if (!mbar_wait(&s_free[s], ((j >> 1) & 1) ^ 1, status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + OFF_K + s * KV_TILE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          umma_bf16(s ? tS1 : tS0, umma_desc_sw128(sQ + (k >> 2) * Q_HALF + (k & 3) * 32),
                    umma_desc_sw128(sK + (k >> 2) * KV_HALF + (k & 3) * 32), IDESC_QK, k > 0 ? 1u : 0u);
        }
        issued = true;
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);      // K_j is no longer needed once S_j is done
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(nkv - 1);
      if (!ok && issued) {
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr, 100000000ull);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int qpos = ctx + q0 + row;  // position in the sequence
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    uint8_t* prow = smem + OFF_P + row * 128;
    const uint32_t swz = (uint32_t)(row & 7);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, status)) { ok = false; break; }
      tc_fence_after();
      uint32_t r[64];
      {
        uint32_t (&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
        uint32_t (&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
        const uint32_t ts = (s ? tS1 : tS0) + lane_off;
        tmem_ld32(ts, r0);
        tmem_ld32(ts + 32, r1);
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(&s_free[s]);  // S[s] is in registers now
      const int key0 = j * BN;
      const bool mask = (key0 + BN - 1 > ctx + q0) || (key0 + BN > total);
      // raw scores stay unscaled: the scale is folded into one FFMA per
      // element below (scale > 0, so the max commutes with it)
      // four independent running maxima, each folding two scores per step
      // (three-input max); only the tiles that cross the diagonal or the
      // sequence end pay for the mask (one compare per score against the
      // row's last valid key), the others take a separate, compare-free loop
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (mask) {
        const int lim = min(qpos + 1, total) - key0;  // keys [0, lim) of the tile are valid for this row
#pragma unroll
        for (int e = 0; e < BN; ++e)
          if (e >= lim) r[e] = __float_as_uint(-INFINITY);
      }
#pragma unroll
      for (int e = 0; e < BN; e += 2)
        mx4[(e >> 1) & 3] = fmaxf(mx4[(e >> 1) & 3], fmaxf(__uint_as_float(r[e]), __uint_as_float(r[e + 1])));
      const float mx_raw = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float mx = mx_raw * scale_log2;
      float m_new = m;
      bool resc = false;
      if (j == 0 || mx > m + RESCALE_THRESHOLD) {  // lazy rescale
        m_new = fmaxf(m, mx);
        resc = (j > 0);
      }
      const float base = (m_new == -INFINITY) ? 0.f : m_new;
      // pairs of elements through packed f32x2 FMA / add (one instruction per
      // two scores); four independent partial sums
      uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[BN / 2];
      const uint64_t sc2 = f32x2(scale_log2, scale_log2), nb2 = f32x2(-base, -base);
#pragma unroll
      for (int e = 0; e < BN; e += 2) {
        const uint64_t t2 = fma_f32x2(f32x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), sc2, nb2);
        // the pair index is a compile-time constant after unrolling: each
        // pair is statically on the special-function unit or the FMA pipe
        uint64_t p2;
        switch ((e >> 1) & 3) {
          case 0: p2 = exp2_pair<EMU, 0>(t2); break;
          case 1: p2 = exp2_pair<EMU, 1>(t2); break;
          case 2: p2 = exp2_pair<EMU, 2>(t2); break;
          default: p2 = exp2_pair<EMU, 3>(t2); break;
        }
        sum2[(e >> 1) & 3] = add_f32x2(sum2[(e >> 1) & 3], p2);
        pk[e >> 1] = pack_bf16x2(lo_f32(p2), hi_f32(p2));
      }
      const uint64_t s01 = add_f32x2(sum2[0], sum2[1]), s23 = add_f32x2(sum2[2], sum2[3]);
      const uint64_t s4 = add_f32x2(s01, s23);
      const float sum = lo_f32(s4) + hi_f32(s4);
      const float alpha = resc ? fast_exp2(m - m_new) : 1.f;
      l = l * alpha + sum;
      m = m_new;
      if (j >= 1) {
        // P smem and O are free once P_{j-1}.V_{j-1} has completed
        if (!mbar_wait(pv_done, (j - 1) & 1, status)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + lane_off + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + lane_off + c * 32, o);
          }
          tmem_st_wait();
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint8_t* dst = prow + ((((uint32_t)c) ^ swz) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      if (PAGED && j == nkv - 1 && total - j * BN < BN) {
        // the last tile's keys past the sequence end are cache slots nobody
        // wrote: their P is 0, but 0 x NaN would still poison O -- zero those
        // V rows (whole 128-byte rows, so the swizzle does not matter)
        if (!mbar_wait(&v_full[s], (j >> 1) & 1, status)) { ok = false; break; }
        uint8_t* vb = smem + OFF_V + s * KV_TILE;
        const int tail = total - j * BN, nz = (BN - tail) * 8;   // 16-byte chunks per half
        for (int t = (int)threadIdx.x - 64; t < 2 * nz; t += 128) {
          const int half = t / nz, rem = t - half * nz;
          *reinterpret_cast<uint4*>(vb + half * KV_HALF + (tail + rem / 8) * 128 + (rem % 8) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();  // P (and zeroed V) stores -> visible to the tensor core
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(pv_done, (nkv - 1) & 1, status)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = q0 + row < seq_len;
      __nv_bfloat16* orow = out + (size_t)(seq_start + q0 + row) * ldo + (size_t)h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + lane_off + c * 32, o);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            u128 w;
            w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            st_v4(orow + c * 32 + v * 8, w);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Two Q tiles per CTA, persistent.  One CTA per SM holds 256 query rows of
// one head as two 128-row tiles X = 0, 1 that share every 128-key K/V tile,
// and the whole tensor memory: S_X = Q_X.K_j^T (128 f32 columns each) and O_X
// (128 each).  P_X is written back over the first 64 columns of S_X as bf16
// pairs and the P.V MMA reads it from there (A operand in tensor memory), so
// the softmax stores nothing to shared memory.  The MMA thread issues, per
// key tile j:
//   P_0.V_j, Q_0.K_{j+1}^T   once softmax 0 has written P_0(j),
//   P_1.V_j, Q_1.K_{j+1}^T   once softmax 1 has written P_1(j),
// so the tensor core runs one tile's P.V and next scores while the other
// tile's softmax runs (the two softmax warpgroups alternate).  The MMAs of
// one thread execute in issue order: Q_X.K_{j+1}^T overwrites S_X only after
// P_X(j).V_j has read it, and the commit of S_X(j+1) also marks P_X(j).V_j
// complete, so the softmax may rescale O_X as soon as it sees S_X(j+1).
// The grid is one CTA per SM; each walks work items (256 query rows x one
// head, heaviest first) in a fixed stride.  The rings and the tensor memory
// carry over: the next item's Q loads as soon as the last Q.K^T of a tile is
// done, its first scores are computed while the softmax warps still store
// the previous item's O, and the next P.V (which overwrites O_X) waits for
// P_X(0) -- which that warpgroup writes only after its epilogue read O_X.
// Warps: 0 TMA producer, 1 MMA issuer (2, 3 idle: warpgroup granularity of
// the register split), 4-7 softmax of tile 0, 8-11 of tile 1 (warp w reaches
// tensor-memory lanes 32 (w % 4) .. + 31).
namespace fap {
constexpr int D = 128;
constexpr int BM = 128;                      // rows of one Q tile
constexpr int BN = 128;                      // keys of one K/V tile
constexpr int ROWS = 2 * BM;                 // query rows of a work item
constexpr int THREADS = 384;                 // three warpgroups
// Registers per thread at launch, and after the setmaxnreg split (no spills).
// 3 warps x 32 x 152 = 14592 of a sub-partition's 16384 leaves 1792: the one
// warp (32 x 48) of a 128-thread KV-push CTA that runs beside this kernel.
constexpr int LAUNCH_REGS = 152;
constexpr int CTRL_REGS = 88, SOFTMAX_REGS = 184;
static_assert(128 * CTRL_REGS + 256 * SOFTMAX_REGS <= THREADS * LAUNCH_REGS, "register split above the launch's total");
constexpr int HALF_Q = BM * 64 * 2;          // [128 rows x 64 dims]: 16 KB
constexpr int HALF_KV = BN * 64 * 2;         // [128 keys x 64 dims]: 16 KB
constexpr int TILE_Q = 2 * HALF_Q;
constexpr int TILE_KV = 2 * HALF_KV;
constexpr int OFF_Q = 0;                     // Q_0, Q_1
constexpr int OFF_K = OFF_Q + 2 * TILE_Q;    // 2 stages
constexpr int OFF_V = OFF_K + 2 * TILE_KV;   // 2 stages
constexpr int OFF_BAR = OFF_V + 2 * TILE_KV;
constexpr int SMEM = OFF_BAR + 256;          // 192.25 KB
constexpr int TMEM_COLS = 512;
constexpr int BPT = BN / 16;                 // paged: 16-token cache blocks per key tile
// Optional per-CTA cycle counters (clock64), 16 per CTA: 0-4 MMA thread waiting
// on q_full / k_full / v_full / p_full[0] / p_full[1], 5 MMA thread total,
// 6-9 and 10-13 softmax warpgroup 0 / 1: waiting on S, softmax (S seen to P
// published), epilogue (O wait + stores), O wait; 14 producer waiting.
constexpr int PROF_SLOTS = 16;
static_assert(SMEM <= 227 * 1024, "shared memory");

// One work item: 256 query rows of a sequence's new tokens, one query head.
struct Item {
  int seq_start, seq_len, q0, ctx, total, h, g, nkv;
  int nt[2];          // key tiles that Q tile X takes part in (0: the tile lies past the sequence end)
  const int* bt;      // paged: the sequence's block table
};
template <bool PAGED>
__device__ __forceinline__ Item item_of(int w, const int* __restrict__ tile_info, int n_tiles, int Hq, int Hkv,
                                        const int* __restrict__ block_tables, int bt_stride) {
  Item it;
  const int tile = w / Hq;   // tile_info lists the heaviest tiles first
  it.h = w - tile * Hq;
  const int* ti = tile_info + tile * (PAGED ? 5 : 3);
  it.seq_start = ti[0];
  it.seq_len = ti[1];
  it.q0 = ti[2];
  it.ctx = PAGED ? ti[3] : 0;
  it.bt = PAGED ? block_tables + (size_t)ti[4] * bt_stride : nullptr;
  it.total = it.ctx + it.seq_len;
  it.g = it.h / (Hq / Hkv);
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int r0 = it.q0 + x * BM;
    it.nt[x] = r0 < it.seq_len ? (min(it.total, it.ctx + r0 + BM) + BN - 1) / BN : 0;
  }
  it.nkv = max(it.nt[0], it.nt[1]);
  return it;
}
// Item of round k for CTA b of G: rounds alternate direction (0..G-1, then
// G-1..0), so over the heaviest-first list every CTA takes alternately
// heavier and lighter positions of consecutive rounds.
__device__ __forceinline__ int item_at(int k, int b, int G) { return k * G + ((k & 1) ? G - 1 - b : b); }
}  // namespace fap

template <bool PAGED, int EMU, bool PROF>
__global__ void __maxnreg__(fap::LAUNCH_REGS)
    prefill_attn_pair_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                             const __grid_constant__ CUtensorMap tmv, __nv_bfloat16* __restrict__ out, int ldo,
                             const int* __restrict__ tile_info, int n_tiles, int Hq, int Hkv, float scale_log2,
                             const int* __restrict__ block_tables, int bt_stride, int* status,
                             unsigned long long* prof) {
  using namespace fap;
  if constexpr (!PROF) prof = nullptr;   // counters compiled out
  using fatc::RESCALE_THRESHOLD;
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0) {  // swizzled operands need a 1 KB-aligned base
    if (threadIdx.x == 0) record_status(status, CX_ERR_BOUNDS);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;    // [tile]
  uint64_t* q_empty = bars + 2;   // [tile]  committed after the item's last Q_X.K^T
  uint64_t* k_full = bars + 4;    // [2 stages]
  uint64_t* k_empty = bars + 6;   // [2]  committed once both tiles' Q.K^T of the stage are done
  uint64_t* v_full = bars + 8;    // [2]
  uint64_t* v_empty = bars + 10;  // [2]  committed once both tiles' P.V of the stage are done
  uint64_t* s_full = bars + 12;   // [tile]  S_X(j) ready
  uint64_t* p_full = bars + 14;   // [tile]  P_X(j) in tensor memory, O_X rescaled (128 arrivals)
  uint64_t* o_full = bars + 16;   // [tile]  O_X of the item final
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  const int n_items = n_tiles * Hq;

  const int warp = warp_id(), lane = lane_id();
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_full[s], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    prefetch_tmap(&tmq);
    if (PAGED) {
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // producer and MMA warps need few registers: hand them to the softmax
    // warpgroups (4 x 32 x 88 + 8 x 32 x 184 = 384 x 152, the launch total)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(CTRL_REGS));
    if (warp == 0) {
      if (lane == 0) {
        bool good = true;
        long long t_wait = 0;
        auto pwait = [&](uint64_t* bar, uint32_t par) -> bool {
          const long long t0 = prof ? clock64() : 0;
          const bool r = mbar_wait(bar, par, status);
          if (prof) t_wait += clock64() - t0;
          return r;
        };
        uint32_t kv = 0;   // key tiles loaded so far: ring position of the item's tile 0
        uint32_t nq[2] = {0u, 0u}, nk[2] = {0u, 0u}, nv[2] = {0u, 0u};   // loads issued per barrier
        for (int n_it = 0, w = item_at(0, blockIdx.x, gridDim.x); w < n_items && good;
             ++n_it, w = item_at(n_it, blockIdx.x, gridDim.x)) {
          const Item it = item_of<PAGED>(w, tile_info, n_tiles, Hq, Hkv, block_tables, bt_stride);
          const int qcol = it.h * D, kcol = (Hq + it.g) * D, vcol = (Hq + Hkv + it.g) * D;
  #pragma unroll
          for (int x = 0; x < 2; ++x) {   // rows past the tensor end are zero-filled, past the sequence unused
            if (!pwait(&q_empty[x], (n_it & 1) ^ 1)) { good = false; break; }
            ++nq[x];
            mbar_arrive_expect_tx(&q_full[x], TILE_Q);
            tma_load_2d(smem + OFF_Q + x * TILE_Q, &tmq, &q_full[x], qcol, it.seq_start + it.q0 + x * BM);
            tma_load_2d(smem + OFF_Q + x * TILE_Q + HALF_Q, &tmq, &q_full[x], qcol + 64,
                        it.seq_start + it.q0 + x * BM);
          }
          if (!good) break;
          // paged: cache rows of the eight 16-token blocks of a key tile (tile j's
          // block ids are fetched one tile ahead so their loads are in flight)
          const int nblk = (it.total + 15) / 16;
          auto rows_of = [&](int j, int (&r)[BPT]) {
  #pragma unroll
            for (int i = 0; i < BPT; ++i) {
              const int b = j * BPT + i;
              r[i] = (it.bt[b < nblk ? b : 0] * Hkv + it.g) * 16;  // past the end: any valid block (masked)
            }
          };
          auto load_tile = [&](const CUtensorMap* map, uint8_t* buf, uint64_t* bar, int col, int j,
                               const int (&r)[BPT]) {
            if constexpr (PAGED) {
  #pragma unroll
              for (int i = 0; i < BPT; ++i) {
                tma_load_2d(buf + i * 2048, map, bar, 0, r[i]);
                tma_load_2d(buf + HALF_KV + i * 2048, map, bar, 64, r[i]);
              }
            } else {
              tma_load_2d(buf, map, bar, col, it.seq_start + j * BN);
              tma_load_2d(buf + HALF_KV, map, bar, col + 64, it.seq_start + j * BN);
            }
          };
          int r_cur[BPT] = {}, r_prev[BPT] = {}, r_next[BPT] = {};
          if (PAGED) rows_of(0, r_cur);
          auto load_k = [&](int j) -> bool {
            const uint32_t u = kv + j, s = u & 1;
            if (!pwait(&k_empty[s], ((u >> 1) & 1) ^ 1)) return false;
            ++nk[s];
            mbar_arrive_expect_tx(&k_full[s], TILE_KV);
            load_tile(&tmk, smem + OFF_K + s * TILE_KV, &k_full[s], kcol, j, r_cur);
            return true;
          };
          auto load_v = [&](int j, const int (&r)[BPT]) -> bool {
            const uint32_t u = kv + j, s = u & 1;
            if (!pwait(&v_empty[s], ((u >> 1) & 1) ^ 1)) return false;
            ++nv[s];
            mbar_arrive_expect_tx(&v_full[s], TILE_KV);
            load_tile(&tmv, smem + OFF_V + s * TILE_KV, &v_full[s], vcol, j, r);
            return true;
          };
          for (int j = 0; j < it.nkv && good; ++j) {   // K_j goes out before V_{j-1}
            good = load_k(j);
            if (PAGED && j + 1 < it.nkv) rows_of(j + 1, r_next);
            if (good && j >= 1) good = load_v(j - 1, r_prev);
  #pragma unroll
            for (int i = 0; i < BPT; ++i) {
              r_prev[i] = r_cur[i];
              r_cur[i] = r_next[i];
            }
          }
          if (good && it.nkv > 0) good = load_v(it.nkv - 1, r_prev);
          kv += it.nkv;
        }
        if (!good) {
          // a wait ran out: let the loads already issued land (bounded) before
          // this CTA can leave, so none writes into shared memory a later CTA owns
          for (int s = 0; s < 2; ++s) {
            if (nq[s]) mbar_wait(&q_full[s], (nq[s] - 1) & 1, nullptr, 100000000ull);
            if (nk[s]) mbar_wait(&k_full[s], (nk[s] - 1) & 1, nullptr, 100000000ull);
            if (nv[s]) mbar_wait(&v_full[s], (nv[s] - 1) & 1, nullptr, 100000000ull);
          }
        }
        if (prof) prof[blockIdx.x * PROF_SLOTS + 14] = (unsigned long long)t_wait;
      }
      __syncwarp();
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t IDESC_QK = umma_idesc_bf16(BM, BN);
        constexpr uint32_t IDESC_PV = umma_idesc_bf16_bmn(BM, D);
        bool ok = true, issued = false;
        long long tw[5] = {0, 0, 0, 0, 0};   // profiling: waits on q_full, k_full, v_full, p_full[0], p_full[1]
        const long long t_start = prof ? clock64() : 0;
        auto mwait = [&](int slot, uint64_t* bar, uint32_t par) -> bool {
          const long long t0 = prof ? clock64() : 0;
          const bool r = mbar_wait(bar, par, status);
          if (prof) tw[slot] += clock64() - t0;
          return r;
        };
        uint32_t kv = 0;               // ring position of the item's tile 0
        uint32_t pf[2] = {0u, 0u};     // p_full phases consumed per tile
        auto qk = [&](int x, uint32_t u) {  // S_x = Q_x.K_u^T, then S_x is signalled
          const uint32_t sQ = smem_u32(smem + OFF_Q + x * TILE_Q);
          const uint32_t sK = smem_u32(smem + OFF_K + (u & 1) * TILE_KV);
  #pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            umma_bf16(tmem + x * BN, umma_desc_sw128(sQ + (k >> 2) * HALF_Q + (k & 3) * 32),
                      umma_desc_sw128(sK + (k >> 2) * HALF_KV + (k & 3) * 32), IDESC_QK, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[x]);
        };
        auto pv = [&](int x, uint32_t u, bool first) {  // O_x (+)= P_x.V_u, P_x in the first 64 columns of S_x
          const uint32_t sV = smem_u32(smem + OFF_V + (u & 1) * TILE_KV);
  #pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            umma_bf16_ts(tmem + 2 * BN + x * D, tmem + x * BN + kk * 8,
                         fatc::umma_desc_sw128_mn(sV + kk * 2048, HALF_KV), IDESC_PV, (!first || kk > 0) ? 1u : 0u);
          }
        };
        for (int n_it = 0, w = item_at(0, blockIdx.x, gridDim.x); w < n_items && ok;
             ++n_it, w = item_at(n_it, blockIdx.x, gridDim.x)) {
          const Item it = item_of<PAGED>(w, tile_info, n_tiles, Hq, Hkv, block_tables, bt_stride);
          for (int x = 0; x < 2 && ok; ++x) ok = mwait(0, &q_full[x], n_it & 1);
          if (!ok) break;
          if (!mwait(1, &k_full[kv & 1], (kv >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
          for (int x = 0; x < 2; ++x) {
            if (it.nt[x] == 0) continue;
            qk(x, kv);
            if (it.nt[x] == 1) umma_commit(&q_empty[x]);   // Q_x done with
          }
          issued = true;
          umma_commit(&k_empty[kv & 1]);
          for (int j = 0; j < it.nkv && ok; ++j) {
            const uint32_t u = kv + j, s = u & 1;
            if (!mwait(2, &v_full[s], (u >> 1) & 1)) { ok = false; break; }
            for (int x = 0; x < 2 && ok; ++x) {
              if (j >= it.nt[x]) continue;
              if (!mwait(3 + x, &p_full[x], pf[x] & 1)) { ok = false; break; }
              ++pf[x];
              tc_fence_after();
              pv(x, u, j == 0);
              if (j + 1 < it.nt[x]) {
                if (!mwait(1, &k_full[(u + 1) & 1], ((u + 1) >> 1) & 1)) { ok = false; break; }
                tc_fence_after();
                qk(x, u + 1);
                if (j + 2 == it.nt[x]) umma_commit(&q_empty[x]);
              } else {
                umma_commit(&o_full[x]);
              }
            }
            if (!ok) break;
            umma_commit(&v_empty[s]);                                  // both tiles' P.V of tile u
            if (j + 1 < it.nkv) umma_commit(&k_empty[(u + 1) & 1]);    // both tiles' Q.K^T of tile u+1
          }
          if (!ok) break;
          for (int x = 0; x < 2; ++x)
            if (it.nt[x] == 0) umma_commit(&q_empty[x]);
          kv += it.nkv;
        }
        if (!ok && issued) {
          umma_commit(drain);
          mbar_wait(drain, 0, nullptr, 100000000ull);
        }
        if (prof) {
          unsigned long long* pr = prof + blockIdx.x * PROF_SLOTS;
          for (int i = 0; i < 5; ++i) pr[i] = (unsigned long long)tw[i];
          pr[5] = (unsigned long long)(clock64() - t_start);
        }
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(SOFTMAX_REGS));
    const int x = (warp >> 2) - 1;        // Q tile of this warpgroup
    const int q = warp & 3;               // its tensor-memory lane quadrant
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t tS = tmem + x * BN + lane_off, tO = tmem + 2 * BN + x * D + lane_off;
    uint32_t sw = 0, ow = 0;              // s_full / o_full phases waited
    uint32_t kv = 0;                      // ring position of the item's tile 0
    bool ok = true;
    const bool rec = prof != nullptr && q == 0 && lane == 0;   // profiling: waits / softmax / epilogue cycles
    long long t_s = 0, t_c = 0, t_e = 0, t_o = 0, t_mark = 0;
    for (int k = 0, w = item_at(0, blockIdx.x, gridDim.x); w < n_items && ok;
         ++k, w = item_at(k, blockIdx.x, gridDim.x)) {
      const Item it = item_of<PAGED>(w, tile_info, n_tiles, Hq, Hkv, block_tables, bt_stride);
      const int r0 = it.q0 + x * BM;      // first query of the tile
      const int qpos = it.ctx + r0 + row; // position in the sequence
      const int n = it.nt[x];
      const int zero_x = it.nt[0] == it.nkv ? 0 : 1;   // the tile whose P.V reads the last V tile first
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        if (rec) t_mark = clock64();
        if (!mbar_wait(&s_full[x], sw & 1, status)) { ok = false; break; }
        ++sw;
        if (rec) {
          const long long t = clock64();
          t_s += t - t_mark;
          t_mark = t;
        }
        tc_fence_after();
        uint32_t r[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
        tmem_ld_wait();
        const int key0 = j * BN;
        // only tiles that cross the diagonal or the sequence end pay for the
        // mask (one compare per score against the row's last valid key)
        const bool mask = (key0 + BN - 1 > it.ctx + r0) || (key0 + BN > it.total);
        if (mask) {
          const int lim = min(qpos + 1, it.total) - key0;  // keys [0, lim) of the tile are valid for this row
#pragma unroll
          for (int e = 0; e < BN; ++e)
            if (e >= lim) r[e] = __float_as_uint(-INFINITY);
        }
        // raw scores stay unscaled (scale > 0 commutes with the max); four
        // independent running maxima, two scores per three-input max
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < BN; e += 2)
          mx4[(e >> 1) & 3] = fmaxf(mx4[(e >> 1) & 3], fmaxf(__uint_as_float(r[e]), __uint_as_float(r[e + 1])));
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale_log2;
        float m_new = m;
        bool resc = false;
        if (j == 0 || mx > m + RESCALE_THRESHOLD) {  // lazy rescale
          m_new = fmaxf(m, mx);
          resc = (j > 0);
        }
        const float base = (m_new == -INFINITY) ? 0.f : m_new;
        uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
        const uint64_t sc2 = f32x2(scale_log2, scale_log2), nb2 = f32x2(-base, -base);
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {   // 32 keys -> 16 bf16 pairs -> 16 columns of S_x
          uint32_t pk[16];
#pragma unroll
          for (int e2 = 0; e2 < 16; ++e2) {
            const int e = c * 32 + 2 * e2;
            const uint64_t t2 = fma_f32x2(f32x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), sc2, nb2);
            if constexpr (EMU == 1) {
              // the pair's exponent rounded to bf16 and one packed ex2 for both
              // (P is stored as bf16 anyway); the row sum stays fp32
              const uint32_t pb = fatc::exp2_bf16x2(pack_bf16x2(lo_f32(t2), hi_f32(t2)));
              sum2[e2 & 3] = add_f32x2(sum2[e2 & 3], f32x2(bf16_lo(pb), bf16_hi(pb)));
              pk[e2] = pb;
            } else {
              uint64_t p2;
              switch (e2 & 3) {   // compile-time after unrolling: each pair's unit is fixed
                case 0: p2 = fatc::exp2_pair<EMU, 0>(t2); break;
                case 1: p2 = fatc::exp2_pair<EMU, 1>(t2); break;
                case 2: p2 = fatc::exp2_pair<EMU, 2>(t2); break;
                default: p2 = fatc::exp2_pair<EMU, 3>(t2); break;
              }
              sum2[e2 & 3] = add_f32x2(sum2[e2 & 3], p2);
              pk[e2] = pack_bf16x2(lo_f32(p2), hi_f32(p2));
            }
          }
          tmem_st16(tS + c * 16, pk);
        }
        const uint64_t s4 = add_f32x2(add_f32x2(sum2[0], sum2[1]), add_f32x2(sum2[2], sum2[3]));
        const float sum = lo_f32(s4) + hi_f32(s4);
        const float alpha = resc ? fatc::fast_exp2(m - m_new) : 1.f;
        l = l * alpha + sum;
        m = m_new;
        if (j >= 1 && __any_sync(0xffffffffu, resc)) {
          // S_x(j) was committed after P_x(j-1).V_{j-1}: O_x is complete here
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
        }
        if (PAGED && x == zero_x && j == it.nkv - 1 && it.total - key0 < BN) {
          // the last tile's keys past the sequence end are cache slots nobody
          // wrote: their P is 0, but 0 x NaN would still poison O -- zero those
          // V rows (whole 128-byte rows, so the swizzle does not matter)
          const uint32_t u = kv + j;
          if (!mbar_wait(&v_full[u & 1], (u >> 1) & 1, status)) { ok = false; break; }
          uint8_t* vb = smem + OFF_V + (u & 1) * TILE_KV;
          const int tail = it.total - key0, nz = (BN - tail) * 8;   // 16-byte chunks per half
          for (int t = q * 32 + lane; t < 2 * nz; t += 128) {
            const int half = t / nz, rem = t - half * nz;
            *reinterpret_cast<uint4*>(vb + half * HALF_KV + (tail + rem / 8) * 128 + (rem % 8) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
        if (rec) t_c += clock64() - t_mark;
      }
      if (!ok) break;
      if (n > 0) {
        const long long te0 = rec ? clock64() : 0;
        if (!mbar_wait(&o_full[x], ow & 1, status)) { ok = false; break; }
        ++ow;
        if (rec) t_o += clock64() - te0;
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const bool valid = r0 + row < it.seq_len;
        __nv_bfloat16* orow = out + (size_t)(it.seq_start + r0 + row) * ldo + (size_t)it.h * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              u128 wv;
              wv.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
              wv.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
              wv.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
              wv.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
              st_v4(orow + c * 32 + v * 8, wv);
            }
          }
        }
        tc_fence_before();   // the next item's P.V overwrites O_x after this warpgroup's next arrival
        if (rec) t_e += clock64() - te0;
      }
      kv += it.nkv;
    }
    if (rec) {
      unsigned long long* pr = prof + blockIdx.x * PROF_SLOTS + 6 + 4 * x;
      pr[0] = (unsigned long long)t_s;
      pr[1] = (unsigned long long)t_c;
      pr[2] = (unsigned long long)t_e;
      pr[3] = (unsigned long long)t_o;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Softmax exponentials: 0 all on ex2.approx.f32; 2 or 4 of every 8 on the
// FMA pipe; 1 (two-tile kernel) one packed bf16x2 ex2 per pair.
static int g_exp_split = 0;
void attention_exp_split(int n) { g_exp_split = n == 1 || n == 2 || n == 4 ? n : 0; }

// Per-CTA cycle counters of the two-tile kernel (0: off), see fap::PROF_SLOTS.
static unsigned long long* g_attn_prof = nullptr;
void attention_profile(int64_t ptr) { g_attn_prof = reinterpret_cast<unsigned long long*>(ptr); }

struct AttnArgs {
  CUtensorMap tq, tk, tv;
  void* out;
  int ldo;
  const int* tile_info;
  int n_tiles, Hq, Hkv;
  float scale_log2;
  const int* bt;
  int bt_stride;
  int* status;
};

// PAIR: the two-tile kernel (256 query rows per CTA, one CTA per SM);
// otherwise the one-tile kernel (128 rows, two CTAs per SM).  PROF: the
// two-tile kernel with its cycle counters.
template <bool PAIR, bool PAGED, int EMU, bool PROF = false>
static void launch_attn(const AttnArgs& a, cudaStream_t s) {
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  auto* kern = PAIR ? prefill_attn_pair_kernel<PAGED, EMU, PROF> : prefill_attn_tc_kernel<PAGED, EMU>;
  const int smem = PAIR ? fap::SMEM : fatc::SMEM;
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr[dev & 63] = true;
  }
  dim3 grid(a.n_tiles, a.Hq);
  if (PAIR) {   // persistent: one CTA per SM over all (tile, head) items
    static int sms[64] = {0};
    if (sms[dev & 63] == 0) cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    grid = dim3(min(a.n_tiles * a.Hq, sms[dev & 63]), 1);
  }
  kern<<<grid, PAIR ? fap::THREADS : fatc::THREADS, smem, s>>>(
      a.tq, a.tk, a.tv, reinterpret_cast<__nv_bfloat16*>(a.out), a.ldo, a.tile_info, a.n_tiles, a.Hq, a.Hkv,
      a.scale_log2, a.bt, a.bt_stride, a.status, PAIR ? g_attn_prof : nullptr);
}

template <bool PAIR, bool PAGED>
static void launch_attn_split(const AttnArgs& a, cudaStream_t s) {
  if (PAIR && g_attn_prof != nullptr)
    launch_attn<PAIR, PAGED, 0, true>(a, s);
  else if (g_exp_split == 1 && PAIR)
    launch_attn<PAIR, PAGED, 1>(a, s);
  else if (g_exp_split == 2)
    launch_attn<PAIR, PAGED, 2>(a, s);
  else if (g_exp_split == 4)
    launch_attn<PAIR, PAGED, 4>(a, s);
  else
    launch_attn<PAIR, PAGED, 0>(a, s);
}

void prefill_attention_tc(const void* qkv, int ldq, int qkv_cols, int T, void* out, int ldo, const int* tile_info,
                          int n_tiles, int Hq, int Hkv, float scale, int* status, cudaStream_t s, int tile_rows) {
  if (n_tiles == 0) return;
  const bool pair = tile_rows == fap::ROWS;
  AttnArgs a;
  a.tq = make_tmap_bf16_2d(qkv, (uint64_t)qkv_cols, (uint64_t)T, (uint64_t)ldq * 2, 64, 128, true);
  a.tk = a.tv = pair ? a.tq : make_tmap_bf16_2d(qkv, (uint64_t)qkv_cols, (uint64_t)T, (uint64_t)ldq * 2, 64, 64, true);
  a.out = out;
  a.ldo = ldo;
  a.tile_info = tile_info;
  a.n_tiles = n_tiles;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.bt = nullptr;
  a.bt_stride = 0;
  a.status = status;
  if (pair)
    launch_attn_split<true, false>(a, s);
  else
    launch_attn_split<false, false>(a, s);
}

void prefill_attention_paged_tc(const void* qkv, int ldq, int qkv_cols, int T, const void* kc, const void* vc,
                                int64_t cache_rows, const int* block_tables, int bt_stride, void* out, int ldo,
                                const int* tile_info, int n_tiles, int Hq, int Hkv, float scale, int* status,
                                cudaStream_t s, int tile_rows) {
  if (n_tiles == 0) return;
  AttnArgs a;
  a.tq = make_tmap_bf16_2d(qkv, (uint64_t)qkv_cols, (uint64_t)T, (uint64_t)ldq * 2, 64, 128, true);
  // caches as [blocks * Hkv * 16 rows, 128 dims]: one row per (block, head, token)
  a.tk = make_tmap_bf16_2d(kc, 128, (uint64_t)cache_rows, 256, 64, 16, true);
  a.tv = make_tmap_bf16_2d(vc, 128, (uint64_t)cache_rows, 256, 64, 16, true);
  a.out = out;
  a.ldo = ldo;
  a.tile_info = tile_info;
  a.n_tiles = n_tiles;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.bt = block_tables;
  a.bt_stride = bt_stride;
  a.status = status;
  if (tile_rows == fap::ROWS)
    launch_attn_split<true, true>(a, s);
  else
    launch_attn_split<false, true>(a, s);
}

}  // namespace cx

// Skinny GEMM for decode steps: D[M,N] = A[M,K] . B[N,K]^T for M <= 8 rows,
// with the epilogues of the tcgen05 GEMM (store, + residual, SiLU(gate) * up).
//
// At M <= 8 every weight byte is used at most 8 times, so the step is bound
// by streaming B from HBM once; a 128-row tensor-core tile would be >= 94 %
// padding and its few output tiles leave most SMs idle or need split-K.
// Here each warp owns 4 weight rows and walks K in 256-element strips: every
// lane issues 4 independent 16-byte non-allocating loads of B per strip (two
// strips in flight), converts bf16 pairs with shifts, and accumulates
// M x 4 fp32 dot products on the CUDA cores; A (a few KB) is read through
// L1 and shared by the 4 rows.  Narrow outputs split K across up to 8 warps
// of a CTA (partials added in shared memory) so every SM keeps ~48 warps of
// loads in flight.  A butterfly reduction gives every lane the sums and
// lanes 0..M-1 write their row's outputs.  For the SiLU-mul
// epilogue a warp's 4 rows are the gate and up rows of two adjacent outputs
// (B is interleaved in 128-row gate / up blocks per 256-row tile).
#include "common.cuh"
#include "gemm.h"

namespace cx {

namespace gv {
constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int ROWS = 4;
constexpr int HALF_TILE = 128;  // gate / up block height of the interleaved gate-up weight
}  // namespace gv

__device__ __forceinline__ void bf16x8_to_f32(const u128& v, float f[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ float gv_silu(float x) { return x / (1.0f + __expf(-x)); }

// KS warps share one group of 4 rows, each taking every KS-th 256-element
// strip of K, and add their partial sums through shared memory: narrow
// outputs (N = 4096) then still put enough loads in flight on every SM.
template <int M, int EPI, int KS>
__global__ void __launch_bounds__(gv::THREADS)
    gemv_bf16_kernel(const __nv_bfloat16* __restrict__ A, int lda, const __nv_bfloat16* __restrict__ B, int ldb,
                     __nv_bfloat16* D, int ldd, const __nv_bfloat16* R, int ldr, int N, int K, int n_groups) {
  using namespace gv;
  __shared__ float part[KS > 1 ? WARPS : 1][ROWS][M];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.x * (WARPS / KS) + warp / KS;
  const int kp = warp % KS;
  const bool live = grp < n_groups;
  if (KS == 1 && !live) return;
  int rows[ROWS];
  if (!live) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) rows[r] = 0;  // idle warp of a K-split CTA: loads nothing (K loop skipped)
  } else if constexpr (EPI == EPI_SILU_MUL) {
    const int o = 2 * grp;                       // outputs o, o + 1
    const int base = (o / HALF_TILE) * (2 * HALF_TILE) + (o % HALF_TILE);
    rows[0] = base;
    rows[1] = base + 1;
    rows[2] = base + HALF_TILE;
    rows[3] = base + HALF_TILE + 1;
  } else {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) rows[r] = min(ROWS * grp + r, N - 1);
  }
  const __nv_bfloat16* brow[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) brow[r] = B + (size_t)rows[r] * ldb;

  float acc[ROWS][M];
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

  auto strip = [&](int k, const u128 (&w)[ROWS]) {
    float wf[ROWS][8];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) bf16x8_to_f32(w[r], wf[r]);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float xf[8];
      bf16x8_to_f32(*reinterpret_cast<const u128*>(A + (size_t)m * lda + k), xf);
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf[r][e], xf[e], acc[r][m]);
    }
  };

  const int kend = live ? K : 0;
  constexpr int STEP = 256 * KS;                 // this warp's strips: kp, kp + KS, ...
  int k = lane * 8 + 256 * kp;
  for (; k + STEP < kend; k += 2 * STEP) {      // two strips in flight
    u128 w0[ROWS], w1[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) w0[r] = ld_nc_v4(brow[r] + k);
#pragma unroll
    for (int r = 0; r < ROWS; ++r) w1[r] = ld_nc_v4(brow[r] + k + STEP);
    strip(k, w0);
    strip(k + STEP, w1);
  }
  if (k < kend) {
    u128 w0[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) w0[r] = ld_nc_v4(brow[r] + k);
    strip(k, w0);
  }

#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      acc[r][m] = v;
    }

  if constexpr (KS > 1) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) part[warp][r][m] = acc[r][m];
    }
    __syncthreads();
    if (kp != 0 || !live) return;
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < KS; ++j) v += part[warp + j][r][m];
        acc[r][m] = v;
      }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    if (lane != m) continue;
    __nv_bfloat16* drow = D + (size_t)m * ldd;
    if constexpr (EPI == EPI_SILU_MUL) {
      const int o = 2 * grp;
      drow[o] = __float2bfloat16(gv_silu(acc[0][m]) * acc[2][m]);
      drow[o + 1] = __float2bfloat16(gv_silu(acc[1][m]) * acc[3][m]);
    } else {
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int n = ROWS * grp + r;
        if (n >= N) break;
        float v = acc[r][m];
        if constexpr (EPI == EPI_ADD) v += __bfloat162float(R[(size_t)m * ldr + n]);
        drow[n] = __float2bfloat16(v);
      }
    }
  }
}

template <int M, int KS>
static void launch_gemv_ks(const __nv_bfloat16* a, int lda, const __nv_bfloat16* b, int ldb, __nv_bfloat16* d,
                           int ldd, const __nv_bfloat16* r, int ldr, int N, int K, int epi, int groups,
                           cudaStream_t s) {
  constexpr int per_cta = gv::WARPS / KS;
  const int ctas = (groups + per_cta - 1) / per_cta;
  if (epi == EPI_SILU_MUL)
    gemv_bf16_kernel<M, EPI_SILU_MUL, KS><<<ctas, gv::THREADS, 0, s>>>(a, lda, b, ldb, d, ldd, r, ldr, N, K, groups);
  else if (epi == EPI_ADD)
    gemv_bf16_kernel<M, EPI_ADD, KS><<<ctas, gv::THREADS, 0, s>>>(a, lda, b, ldb, d, ldd, r, ldr, N, K, groups);
  else
    gemv_bf16_kernel<M, EPI_STORE, KS><<<ctas, gv::THREADS, 0, s>>>(a, lda, b, ldb, d, ldd, r, ldr, N, K, groups);
}

template <int M>
static void launch_gemv(const void* A, const void* B, void* D, const void* R, int N, int K, int lda, int ldb, int ldd,
                        int ldr, int epi, cudaStream_t s) {
  auto a = reinterpret_cast<const __nv_bfloat16*>(A);
  auto b = reinterpret_cast<const __nv_bfloat16*>(B);
  auto d = reinterpret_cast<__nv_bfloat16*>(D);
  auto r = reinterpret_cast<const __nv_bfloat16*>(R);
  const int groups = epi == EPI_SILU_MUL ? N / 4 : (N + gv::ROWS - 1) / gv::ROWS;
  // enough warps for ~48 per SM, each with at least two 256-element strips of K
  const long want = 48L * num_sms();
  int ks = 1;
  while (ks < gv::WARPS && (long)groups * ks < want && K >= 2 * 256 * (ks * 2)) ks *= 2;
  switch (ks) {
    case 1: launch_gemv_ks<M, 1>(a, lda, b, ldb, d, ldd, r, ldr, N, K, epi, groups, s); break;
    case 2: launch_gemv_ks<M, 2>(a, lda, b, ldb, d, ldd, r, ldr, N, K, epi, groups, s); break;
    case 4: launch_gemv_ks<M, 4>(a, lda, b, ldb, d, ldd, r, ldr, N, K, epi, groups, s); break;
    default: launch_gemv_ks<M, 8>(a, lda, b, ldb, d, ldd, r, ldr, N, K, epi, groups, s); break;
  }
}

bool gemv_bf16_tn(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb, int ldd,
                  int ldr, int epi, cudaStream_t s) {
  if (M < 1 || M > GEMV_MAX_M) return false;
  if (epi == EPI_SILU_MUL && N % (2 * gv::HALF_TILE) != 0) return false;
  switch (M) {  // exact row counts: a rounded-up M would read and write rows that do not exist
    case 1: launch_gemv<1>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    case 2: launch_gemv<2>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    case 3: launch_gemv<3>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    case 4: launch_gemv<4>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    case 5: launch_gemv<5>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    case 6: launch_gemv<6>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    case 7: launch_gemv<7>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
    default: launch_gemv<8>(A, B, D, R, N, K, lda, ldb, ldd, ldr, epi, s); break;
  }
  return true;
}

}  // namespace cx

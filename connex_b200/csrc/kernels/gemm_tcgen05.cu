// Persistent bf16 GEMM on the sm_100a 5th-generation tensor cores.
//
//   D[M, N] = A[M, K] . B[N, K]^T      (both operands K-major, fp32 accumulate)
//
// This is the dense-layer GEMM of the serving runtime (a torch Linear weight
// is already [out, in] = [N, K]).  Design, per CTA (one CTA per SM):
//   warp 0      : TMA producer.  128x64 A and BNx64 B boxes, 128-byte swizzle,
//                 STAGES-deep ring of shared-memory stages (no cluster multicast).
//   warp 1      : allocates TMEM (2 accumulators x BN fp32 columns) and one
//                 elected thread issues tcgen05.mma (M=128, N=BN, K=16) and
//                 tcgen05.commit to release stages / publish accumulators.
//   warps 2..5  : epilogue.  tcgen05.ld 32 columns at a time from the TMEM lane
//                 quadrant the warp owns, fuse (residual add | SiLU(gate)*up),
//                 convert to bf16 and store.  The second accumulator lets the
//                 epilogue of tile i overlap the MMAs of tile i+1.
// Tiles are visited in a grouped raster (16 tile-rows per band) so that one
// wave of CTAs shares A and B tiles through the 126 MB L2.
//
// Every mbarrier wait is bounded (see common.cuh); a timeout writes a status
// code and the CTA drains its tensor-core work before freeing TMEM.
#include "common.cuh"
#include "gemm.h"

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

namespace cx {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

template <int BN, int STAGES>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
  static constexpr int SMEM = 1024 /*align slack*/ + STAGES * STAGE_BYTES + 256 /*barriers*/;
};

// Grouped raster: bands of `group` tile-rows, each band walked column by
// column, so the CTAs of one wave share A rows and B columns through L2.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group, int& tm, int& tn) {
  const int per_group = group * num_n;
  const int g = t / per_group;
  const int first_m = g * group;
  const int gm = min(num_m - first_m, group);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ void tile_coords_split(int t, int num_m, int num_n, int splits, int group, int& tm,
                                                  int& tn, int& ks) {
  const int tt = t / splits;
  ks = t - tt * splits;
  tile_coords(tt, num_m, num_n, group, tm, tn);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Vector fp32 reduction into global memory (split-K partial sums).
__device__ __forceinline__ void red_add_v4_f32(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// SPLIT: the K loop of each output tile is cut into `splits` chunks of `kper`
// k-blocks, one work item each, and the epilogue adds the fp32 partial sums
// into W (zero on entry) with vector reductions; gemm_splitk_finalize applies
// the epilogue.  Small-M (decode) GEMMs get enough work items to fill the SMs.
// Tile-rows per raster band (see tile_coords).  Measured on one B200 (bands of
// 4 / 8 / 16 / 32): 8192^3 0.80 / 0.84 / 0.86 / 0.85 of the cuBLAS burst peak,
// 8192 x 28672 x 4096 with the SiLU epilogue 0.70 / 0.73 / 0.75 / 0.76.
static int g_gemm_group = 16;
void gemm_raster_group(int rows) { g_gemm_group = rows >= 1 && rows <= 64 ? rows : 16; }

template <int BN, int STAGES, int EPI, bool SPLIT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        __nv_bfloat16* __restrict__ D, const __nv_bfloat16* R, int M, int N, int K, int ldd,
                        int ldr, int* status, float* __restrict__ W, int ldw, int splits, int kper, int group) {
  using Cfg = GemmCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = (N + BN - 1) / BN;
  const int total = num_m * num_n * splits;
  const int nk = (K + GEMM_BK - 1) / GEMM_BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int tm, tn, ks;
        tile_coords_split(t, num_m, num_n, splits, group, tm, tn, ks);
        const int kb0 = ks * kper, kb1 = min(nk, kb0 + kper);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * GEMM_BK, tm * GEMM_BM);
          tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * GEMM_BK, tn * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let loads already in flight land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full[s], 0, nullptr, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = umma_idesc_bf16(GEMM_BM, BN);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        const int ks = t % splits;
        const int kb0 = ks * kper, kb1 = min(nk, kb0 + kper);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            umma_bf16(d, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), IDESC,
                      (kb != kb0 || k != 0) ? 1u : 0u);
          }
          issued = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (!ok && issued) {
        // Drain: wait (bounded) for every issued MMA before TMEM is freed.
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr, 100000000ull);
      }
    }
    __syncwarp();
  } else {
    // Epilogue warps 2..5 -> TMEM lane quadrants 2,3,0,1.
    const int q = warp & 3;
    uint32_t acc = 0, acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int tm, tn, ks;
      tile_coords_split(t, num_m, num_n, splits, group, tm, tn, ks);
      if (!mbar_wait(&tfull[acc], acc_phase, status)) break;
      tc_fence_after();
      const int row = tm * GEMM_BM + q * 32 + lane;
      const uint32_t tb = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if constexpr (SPLIT) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tb + c * 32, r);
          tmem_ld_wait();
          const int col = tn * BN + c * 32;
          if (row < M) {
            float* dst = W + (size_t)row * ldw + col;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              if (col + v * 4 < N)
                red_add_v4_f32(dst + v * 4, __uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                               __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          }
        }
      } else if constexpr (EPI == EPI_SILU_MUL) {
        constexpr int HALF = BN / 2;
#pragma unroll 1
        for (int c = 0; c < HALF / 32; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(tb + c * 32, g);
          tmem_ld32(tb + HALF + c * 32, u);
          tmem_ld_wait();
          const int col = tn * HALF + c * 32;
          if (row < M) {
            u128 out[4];
            uint32_t* o = reinterpret_cast<uint32_t*>(out);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float a0 = silu(__uint_as_float(g[2 * j])) * __uint_as_float(u[2 * j]);
              float a1 = silu(__uint_as_float(g[2 * j + 1])) * __uint_as_float(u[2 * j + 1]);
              o[j] = pack_bf16x2(a0, a1);
            }
            __nv_bfloat16* dst = D + (size_t)row * ldd + col;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < N / 2) st_v4(dst + v * 8, out[v]);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tb + c * 32, r);
          tmem_ld_wait();
          const int col = tn * BN + c * 32;
          if (row < M) {
            u128 out[4];
            uint32_t* o = reinterpret_cast<uint32_t*>(out);
            if constexpr (EPI == EPI_ADD) {
              const __nv_bfloat16* src = R + (size_t)row * ldr + col;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                u128 rv = (col + v * 8 < N) ? ld_v4(src + v * 8) : u128{0, 0, 0, 0};
                const uint32_t* rr = reinterpret_cast<const uint32_t*>(&rv);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  float a0 = __uint_as_float(r[v * 8 + 2 * j]) + bf16_lo(rr[j]);
                  float a1 = __uint_as_float(r[v * 8 + 2 * j + 1]) + bf16_hi(rr[j]);
                  o[v * 4 + j] = pack_bf16x2(a0, a1);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) o[j] = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            }
            __nv_bfloat16* dst = D + (size_t)row * ldd + col;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < N) st_v4(dst + v * 8, out[v]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// D = epilogue(W) for a split-K GEMM; W is read once and left zero for the next call.
template <int EPI>
__global__ void __launch_bounds__(256) gemm_splitk_finalize(float* __restrict__ W, int ldw, __nv_bfloat16* D, int ldd,
                                                            const __nv_bfloat16* R, int ldr, int M, int Nout) {
  const int per_row = Nout / 8;
  const long total = (long)M * per_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int row = (int)(i / per_row), c8 = (int)(i - (long)row * per_row) * 8;
    float v[8];
    float* w = W + (size_t)row * ldw;
    if constexpr (EPI == EPI_SILU_MUL) {
      const int base = (c8 / 128) * 256 + (c8 % 128);   // gate / up rows interleaved per 256-wide tile
      float4* g = reinterpret_cast<float4*>(w + base);
      float4* u = reinterpret_cast<float4*>(w + base + 128);
      const float4 g0 = g[0], g1 = g[1], u0 = u[0], u1 = u[1];
      const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = silu(gg[j]) * uu[j];
      g[0] = g[1] = u[0] = u[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      float4* p = reinterpret_cast<float4*>(w + c8);
      const float4 a = p[0], b = p[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      p[0] = p[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (EPI == EPI_ADD) {
        const u128 rv = ld_v4(R + (size_t)row * ldr + c8);
        const uint32_t* rr = reinterpret_cast<const uint32_t*>(&rv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] += bf16_lo(rr[j]);
          v[2 * j + 1] += bf16_hi(rr[j]);
        }
      }
    }
    u128 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    st_v4(D + (size_t)row * ldd + c8, o);
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cx: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("cx: TMA base not 16-byte aligned");
  if ((row_stride_bytes & 15) != 0) throw std::runtime_error("cx: TMA row stride not a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cx: cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int STAGES, int EPI, bool SPLIT = false>
static void launch_gemm(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb,
                        int ldd, int ldr, int* status, int max_ctas, cudaStream_t stream, float* W = nullptr,
                        int splits = 1, int kper = 0) {
  using Cfg = GemmCfg<BN, STAGES>;
  auto kern = gemm_bf16_tn_kernel<BN, STAGES, EPI, SPLIT>;
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set[dev & 63] = true;
  }
  CUtensorMap ta = make_tmap_bf16_2d(A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, GEMM_BK, GEMM_BM, true);
  CUtensorMap tb = make_tmap_bf16_2d(B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * 2, GEMM_BK, BN, true);
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN) * splits;
  int grid = tiles < num_sms() ? tiles : num_sms();
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  if (kper <= 0) kper = (K + GEMM_BK - 1) / GEMM_BK;
  kern<<<grid, GEMM_THREADS, Cfg::SMEM, stream>>>(ta, tb, reinterpret_cast<__nv_bfloat16*>(D),
                                                   reinterpret_cast<const __nv_bfloat16*>(R), M, N, K, ldd, ldr,
                                                   status, W, N, splits, kper, g_gemm_group);
}

// Work-item split of the K loop: only when the output tiles alone would
// leave most SMs idle (small-M decode GEMMs) and K is long enough.
int gemm_splits(int M, int N, int K, int epi, int bn) {
  if (bn == 0 && M <= GEMV_MAX_M) return 1;  // the skinny kernel takes these
  if (bn == 0) bn = epi == EPI_SILU_MUL ? 256 : 128;
  const long tiles = (long)((M + GEMM_BM - 1) / GEMM_BM) * ((N + bn - 1) / bn);
  const int nk = (K + GEMM_BK - 1) / GEMM_BK;
  const int sms = num_sms();
  if (tiles * 2 > sms || nk < 8) return 1;
  int s = (int)(sms / tiles);
  if (s > nk / 4) s = nk / 4;
  if (s < 2) return 1;
  const int kper = (nk + s - 1) / s;
  return (nk + kper - 1) / kper;  // no empty split
}

void gemm_bf16_tn(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb,
                  int ldd, int ldr, int epi, int bn, int* status, int max_ctas, cudaStream_t stream, float* W,
                  int splits) {
  if (K % 8 != 0) throw std::runtime_error("cx gemm: K must be a multiple of 8");
  if ((lda | ldb | ldd) % 8 != 0 || (R != nullptr && ldr % 8 != 0))
    throw std::runtime_error("cx gemm: leading dimensions must be multiples of 8 elements");
  if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)D | (uintptr_t)R) & 15)
    throw std::runtime_error("cx gemm: operands must be 16-byte aligned");
  if (N % 8 != 0) throw std::runtime_error("cx gemm: N must be a multiple of 8");
  if (bn == 0 && max_ctas == 0 && splits <= 1 && M <= GEMV_MAX_M &&
      gemv_bf16_tn(A, B, D, R, M, N, K, lda, ldb, ldd, ldr, epi, stream))
    return;
  if (bn == 0) {
    // Prefer 256-wide tiles unless that leaves most SMs idle.
    const long tiles256 = (long)((M + 127) / 128) * ((N + 255) / 256);
    bn = (tiles256 >= num_sms() || N <= 128) ? 256 : 128;
    if (epi == EPI_SILU_MUL) bn = 256;
  }
  if (epi == EPI_SILU_MUL && (N % bn) != 0)
    throw std::runtime_error("cx gemm: SiLU-mul epilogue needs N to be a multiple of the tile width");
  if (splits > 1) {
    if (W == nullptr || ((uintptr_t)W & 15)) throw std::runtime_error("cx gemm: split-K needs a 16-byte aligned workspace");
    const int sbn = epi == EPI_SILU_MUL ? 256 : 128;
    const int nk = (K + GEMM_BK - 1) / GEMM_BK;
    const int kper = (nk + splits - 1) / splits;
    splits = (nk + kper - 1) / kper;
    if (sbn == 256)
      launch_gemm<256, 4, EPI_STORE, true>(A, B, D, R, M, N, K, lda, ldb, ldd, ldr, status, max_ctas, stream, W,
                                           splits, kper);
    else
      launch_gemm<128, 6, EPI_STORE, true>(A, B, D, R, M, N, K, lda, ldb, ldd, ldr, status, max_ctas, stream, W,
                                           splits, kper);
    const int Nout = epi == EPI_SILU_MUL ? N / 2 : N;
    const long chunks = (long)M * (Nout / 8);
    const int blocks = (int)std::min<long>((chunks + 255) / 256, (long)num_sms() * 8);
    auto* d = reinterpret_cast<__nv_bfloat16*>(D);
    auto* r = reinterpret_cast<const __nv_bfloat16*>(R);
    if (epi == EPI_SILU_MUL)
      gemm_splitk_finalize<EPI_SILU_MUL><<<blocks, 256, 0, stream>>>(W, N, d, ldd, r, ldr, M, Nout);
    else if (epi == EPI_ADD)
      gemm_splitk_finalize<EPI_ADD><<<blocks, 256, 0, stream>>>(W, N, d, ldd, r, ldr, M, Nout);
    else
      gemm_splitk_finalize<EPI_STORE><<<blocks, 256, 0, stream>>>(W, N, d, ldd, r, ldr, M, Nout);
    return;
  }
#define CX_GEMM_CASE(BNV, ST, E)                                                                   \
  if (bn == BNV && epi == E) {                                                                     \
    launch_gemm<BNV, ST, E>(A, B, D, R, M, N, K, lda, ldb, ldd, ldr, status, max_ctas, stream); \
    return;                                                                                        \
  }
  CX_GEMM_CASE(256, 4, EPI_STORE)
  CX_GEMM_CASE(256, 4, EPI_ADD)
  CX_GEMM_CASE(256, 4, EPI_SILU_MUL)
  CX_GEMM_CASE(128, 6, EPI_STORE)
  CX_GEMM_CASE(128, 6, EPI_ADD)
  CX_GEMM_CASE(128, 6, EPI_SILU_MUL)
#undef CX_GEMM_CASE
  throw std::runtime_error("cx gemm: unsupported tile width / epilogue");
}

}  // namespace cx

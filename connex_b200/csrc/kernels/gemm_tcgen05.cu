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
// Tiles are visited in a grouped raster (8 tile-rows per band) so that one
// wave of CTAs shares A and B tiles through the 126 MB L2.
//
// Every mbarrier wait is bounded (see common.cuh); a timeout writes a status
// code and the CTA drains its tensor-core work before freeing TMEM.
#include "common.cuh"
#include "gemm.h"

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

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  constexpr int GROUP = 8;
  const int per_group = GROUP * num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP;
  const int gm = min(num_m - first_m, GROUP);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        __nv_bfloat16* __restrict__ D, const __nv_bfloat16* R, int M, int N, int K, int ldd,
                        int ldr, int* status) {
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
  const int total = num_m * num_n;
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
        int tm, tn;
        tile_coords(t, num_m, num_n, tm, tn);
        for (int kb = 0; kb < nk; ++kb) {
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
        for (int kb = 0; kb < nk; ++kb) {
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
                      (kb | k) != 0 ? 1u : 0u);
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
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, status)) break;
      tc_fence_after();
      const int row = tm * GEMM_BM + q * 32 + lane;
      const uint32_t tb = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if constexpr (EPI == EPI_SILU_MUL) {
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

template <int BN, int STAGES, int EPI>
static void launch_gemm(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb,
                        int ldd, int ldr, int* status, int max_ctas, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, STAGES>;
  auto kern = gemm_bf16_tn_kernel<BN, STAGES, EPI>;
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set[dev & 63] = true;
  }
  CUtensorMap ta = make_tmap_bf16_2d(A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, GEMM_BK, GEMM_BM, true);
  CUtensorMap tb = make_tmap_bf16_2d(B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * 2, GEMM_BK, BN, true);
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN);
  int grid = tiles < num_sms() ? tiles : num_sms();
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  kern<<<grid, GEMM_THREADS, Cfg::SMEM, stream>>>(ta, tb, reinterpret_cast<__nv_bfloat16*>(D),
                                                   reinterpret_cast<const __nv_bfloat16*>(R), M, N, K, ldd, ldr,
                                                   status);
}

void gemm_bf16_tn(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb,
                  int ldd, int ldr, int epi, int bn, int* status, int max_ctas, cudaStream_t stream) {
  if (K % 8 != 0) throw std::runtime_error("cx gemm: K must be a multiple of 8");
  if ((lda | ldb | ldd) % 8 != 0 || (R != nullptr && ldr % 8 != 0))
    throw std::runtime_error("cx gemm: leading dimensions must be multiples of 8 elements");
  if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)D | (uintptr_t)R) & 15)
    throw std::runtime_error("cx gemm: operands must be 16-byte aligned");
  if (N % 8 != 0) throw std::runtime_error("cx gemm: N must be a multiple of 8");
  if (bn == 0) {
    // Prefer 256-wide tiles unless that leaves most SMs idle.
    const long tiles256 = (long)((M + 127) / 128) * ((N + 255) / 256);
    bn = (tiles256 >= num_sms() || N <= 128) ? 256 : 128;
    if (epi == EPI_SILU_MUL) bn = 256;
  }
  if (epi == EPI_SILU_MUL && (N % bn) != 0)
    throw std::runtime_error("cx gemm: SiLU-mul epilogue needs N to be a multiple of the tile width");
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

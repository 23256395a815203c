// Host-side entry points of the tcgen05 GEMM (gemm_tcgen05.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cx {

enum GemmEpilogue : int {
  EPI_STORE = 0,     // D = A.B^T
  EPI_ADD = 1,       // D = A.B^T + R          (R may alias D: in-place residual)
  EPI_SILU_MUL = 2,  // D[:, j] = SiLU(acc[:, g(j)]) * acc[:, u(j)], B rows interleaved per tile
};

// D[M,N] (ld ldd) = A[M,K] (ld lda) . B[N,K]^T (ld ldb); bf16 in/out, fp32 accumulate.
// bn = 0 picks the tile width.  status: int32 device word (0 = ok).
// splits > 1: split-K into W (fp32 [M, N], zero on entry, left zero) + a finalize kernel.
void gemm_bf16_tn(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb,
                  int ldd, int ldr, int epi, int bn, int* status, int max_ctas, cudaStream_t stream,
                  float* W = nullptr, int splits = 1);
// The K split gemm_bf16_tn would profit from (1 = none).
int gemm_splits(int M, int N, int K, int epi, int bn);
// Tile-rows per band of the GEMM's grouped raster (default 16).
void gemm_raster_group(int rows);

// M <= GEMV_MAX_M rows (decode steps): the weight-streaming CUDA-core kernel
// (gemv.cu) that gemm_bf16_tn dispatches to when bn, max_ctas and splits are
// left to it; returns false for shapes it does not take.
constexpr int GEMV_MAX_M = 8;
bool gemv_bf16_tn(const void* A, const void* B, void* D, const void* R, int M, int N, int K, int lda, int ldb, int ldd,
                  int ldr, int epi, cudaStream_t s);

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer, bool swizzle128);
int num_sms();

}  // namespace cx

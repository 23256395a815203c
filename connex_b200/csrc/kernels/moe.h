// Host entry points of the expert-parallel MoE kernels (moe.cu).
//
// One MoE layer on rank `me` of N (S expert slots per rank, top-K routing):
//   ep_count     -> counts[N][N][S] broadcast to every rank + count flags
//   ep_dispatch  -> token rows + metadata into the owners' receive buffers
//   ep_grouped_gemm (gate/up, SiLU-mul)   local
//   ep_grouped_gemm (down, combine store) -> weighted rows into the sources'
//                                            combine buffers + combine flags
//   ep_combine   -> y[t] = sum_k comb[t][k]
// Peer addresses are passed as device arrays of N uint64 (this rank's entry
// is its own local address).  Flags are u32 counters compared cyclically.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace cx {

struct EpPeers {
  const uint64_t* counts;     // [N] -> int32 [N][N][S] count matrix on each rank
  const uint64_t* count_flag; // [N] -> u32 count flag on each rank
  const uint64_t* recv;       // [N] -> bf16 [R_max][H] receive buffer on each rank
  const uint64_t* recv_meta;  // [N] -> int4 [R_max] (src, t*K+k, weight bits, 0) on each rank
  const uint64_t* data_flag;  // [N] -> u32 data flag on each rank
  const uint64_t* comb;       // [N] -> bf16 [T_max*K][H] combine buffer on each rank
  const uint64_t* comb_flag;  // [N] -> u32 combine flag on each rank
};

constexpr int EP_DISPATCH_CTAS = 132;
constexpr int EP_MAX_RANKS = 64;

// Count kernel: one CTA.  pos[T*K] receives each routed row's index in its
// (dst rank, slot) bucket, slot_of[T*K] its global physical slot (-1: not
// routable, e.g. no live replica).  Adds (valid rows x arrivals_per_row) to
// *comb_expect and 1 to every rank's count flag when done.
void ep_count(const int* topk_idx, const int* l2p, const int* l2p_cnt, int max_rep, int T, int K, int N, int S,
              int me, int* pos, int* slot_of, EpPeers peers, uint32_t* comb_expect, int arrivals_per_row, int* status,
              cudaStream_t s);

// Dispatch kernel: waits until the local count flag reaches count_target,
// then scatters.  Adds 1 to every rank's data flag per CTA (EP_DISPATCH_CTAS).
void ep_dispatch(const void* x, const float* topk_w, const int* pos, const int* slot_of, const int* counts_local,
                 int T, int K, int H, int N, int S, int me, int R_max, uint32_t count_target, EpPeers peers,
                 int* status, cudaStream_t s);

// Grouped GEMM over the S local experts.  Rows of expert e are
// [seg(e), seg(e+1)) of A where seg comes from the local count matrix.
//   mode 0: D[row] = SiLU(gate) * up   (B = w13 [S][2F][K] interleaved per 256-row tile)
//   mode 1: combine store: row r with meta (src, tk, w) ->
//           comb[src][tk][:] = w * (A[r] . B_e^T), then +1 on comb_flag[src]
// wait_target: the kernel first waits until *wait_flag reaches it.
void ep_grouped_gemm(const void* A, int lda, const void* B, int n_per_expert, int K, void* D, int ldd,
                     const int* counts_local, int N, int S, int me, int R_max, int mode, const int* recv_meta,
                     EpPeers peers, int H, const uint32_t* wait_flag, uint32_t wait_target, int* status,
                     cudaStream_t s);

// Combine: waits until the local comb flag reaches *expect, then
// y[t] = sum over routable k of comb[t*K+k].
void ep_combine(const void* comb, const int* slot_of, int T, int K, int H, void* y, const uint32_t* comb_flag,
                const uint32_t* expect, int* status, cudaStream_t s);

}  // namespace cx

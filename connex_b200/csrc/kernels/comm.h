// Host entry points of the peer-memory kernels (kv_push.cu, moe.cu, wsync.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdexcept>

namespace cx {

int num_sms_comm();

// Returns the number of CTAs launched (each releases `ready` by one).
// `span` (optional, 2 x u64 initialised to {UINT64_MAX, 0}): receives the
// kernel's execution window in %globaltimer nanoseconds.  `threads` per CTA:
// 256, or 128 for a push that runs beside the prefill's persistent kernels
// (one 128-thread CTA fits in the registers they leave free on each SM).
int kv_push_layer(const void* src_k, const void* src_v, void* dst_k, void* dst_v, const int* pairs, int n_pairs,
                  int src_heads, int dst_heads, int src_h0, int dst_h0, int n_heads, int chunk_bytes, int src_blocks,
                  int dst_blocks, uint32_t* ready, int max_ctas, int* status, cudaStream_t s,
                  uint64_t* span = nullptr, int threads = 256);

int copy_segments(const int64_t* segs, int n, int64_t total_bytes, uint32_t* ready, int max_ctas, int* status,
                  cudaStream_t s);

// Weight sync (wsync.cu): fused cast + re-layout broadcast.  Returns the CTA
// count; each CTA releases +1 on every destination flag when it is done.
constexpr int WS_JOB_COLS = 12;
constexpr int WS_MAX_DST = 8;
int wsync(const int64_t* jobs_dev, const int64_t* jobs_host, int n_jobs, int64_t dst_bytes, const uint64_t* dst_bases,
          const uint64_t* dst_flags, int n_dst, uint64_t mc_base, uint64_t mc_flag, int max_ctas, int64_t scatter_bytes, cudaStream_t s);

// P2P channel copy (chan.cu): wait, copy up to CH_MAX_SEGS segments, signal
// (mode 1: +1 per CTA on `signal`; mode 2: the last CTA stores `value`).
// `abort` (may be null): pinned host word; nonzero = the peer is gone, do nothing.
constexpr int CH_MAX_SEGS = 8;
void chan_copy(const uint64_t* src, const uint64_t* dst, const uint64_t* bytes, int n, const uint32_t* wait_on,
               uint32_t wait_target, uint64_t timeout_ns, const uint32_t* abort, uint32_t* signal, uint32_t value,
               int mode, uint32_t* done_ctr, int ctas, int* status, cudaStream_t s);

void wait_flag(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status, cudaStream_t s);
void write_flag(uint32_t* flag, uint32_t value, bool add, cudaStream_t s);

}  // namespace cx

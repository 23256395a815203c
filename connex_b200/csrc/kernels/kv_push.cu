// Peer-memory data movement kernels.
//
// kv_push_layer : the prefill -> decode paged-KV transfer of one layer.
//   For every (source block, destination block) pair of the requests whose
//   prefill has written layer l, each warp moves one 4 KB head-slice
//   ([BS=16 tokens x 128 dims] bf16, contiguous in the [blocks, Hkv, BS, D]
//   cache) from this GPU's cache straight into the decode GPU's cache through
//   its NVLink peer mapping (16-byte loads, 8 in flight per lane, streaming
//   stores).  A head range re-layout (src heads [sh0, sh0+nh) -> dst heads
//   [dh0, dh0+nh)) covers prefill/decode instances with different TP degrees.
//   When all of its stores are issued a CTA releases (+1, system scope) the
//   decode side's ready counter, so the decode stream can acquire-wait on it
//   without any host round trip.  Launched on a side stream right after the
//   layer's KV is written, it overlaps the remaining prefill layers.
//
// copy_segments : batched (src, dst, bytes) copy with the same completion
//   signal; used for expert-weight migration, one-sided reads of registered
//   regions and the weight-sync peer-pull fallback.
//
// wait_flag / write_flag : stream-ordered, bounded device waits and
//   release stores on u32 counters (cyclic compare), the device side of the
//   GPU-driven channels.
#include "common.cuh"
#include "comm.h"

namespace cx {

__device__ __forceinline__ void signal_done(uint32_t* flag) {
  __syncthreads();
  if (threadIdx.x == 0 && flag != nullptr) {
    __threadfence_system();
    red_release_sys_add_u32(flag, 1u);
  }
}

__global__ void __launch_bounds__(256) kv_push_kernel(const uint8_t* __restrict__ sk, const uint8_t* __restrict__ sv,
                                                      uint8_t* dk, uint8_t* dv, const int* __restrict__ pairs,
                                                      int n_pairs, int sH, int dH, int sh0, int dh0, int nh,
                                                      int chunk_bytes, int src_blocks, int dst_blocks,
                                                      uint32_t* ready, int* status,
                                                      unsigned long long* span) {
  // span (optional): [first CTA start, last CTA end] in %globaltimer ns -- the
  // kernel's own execution window, free of launch and queueing delays
  if (span != nullptr && threadIdx.x == 0) atomicMin(&span[0], (unsigned long long)globaltimer_ns());
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const long total = (long)n_pairs * 2 * nh;
  const int vec_per_lane = chunk_bytes / (16 * 32);  // 8 for 4 KB chunks
  for (long c = (long)blockIdx.x * wpb + (threadIdx.x >> 5); c < total; c += (long)gridDim.x * wpb) {
    const int h = (int)(c % nh);
    const long pk = c / nh;
    const int kv = (int)(pk & 1);
    const int p = (int)(pk >> 1);
    const int sb = pairs[2 * p], db = pairs[2 * p + 1];
    if (sb < 0 || sb >= src_blocks || db < 0 || db >= dst_blocks) {
      record_status(status, CX_ERR_BOUNDS);
      continue;
    }
    const uint8_t* src = (kv ? sv : sk) + ((size_t)sb * sH + sh0 + h) * chunk_bytes;
    uint8_t* dst = (kv ? dv : dk) + ((size_t)db * dH + dh0 + h) * chunk_bytes;
    if (vec_per_lane == 8) {
      u128 r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = ld_nc_v4(src + (i * 32 + lane) * 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) st_cs_v4(dst + (i * 32 + lane) * 16, r[i]);
    } else {
      for (int i = lane; i < chunk_bytes / 16; i += 32) st_cs_v4(dst + i * 16, ld_nc_v4(src + i * 16));
    }
  }
  signal_done(ready);
  if (span != nullptr && threadIdx.x == 0) atomicMax(&span[1], (unsigned long long)globaltimer_ns());
}

int kv_push_layer(const void* src_k, const void* src_v, void* dst_k, void* dst_v, const int* pairs, int n_pairs,
                  int src_heads, int dst_heads, int src_h0, int dst_h0, int n_heads, int chunk_bytes, int src_blocks,
                  int dst_blocks, uint32_t* ready, int max_ctas, int* status, cudaStream_t s, uint64_t* span,
                  int threads) {
  if (n_pairs <= 0) return 0;
  if (chunk_bytes % 16 != 0) throw std::runtime_error("cx kv_push: head slice must be a multiple of 16 bytes");
  if (threads != 128 && threads != 256) throw std::runtime_error("cx kv_push: 128 or 256 threads per CTA");
  const long warps = (long)n_pairs * 2 * n_heads;
  const int wpb = threads / 32;
  long ctas = (warps + wpb - 1) / wpb;
  const long cap = max_ctas > 0 ? max_ctas : 4L * num_sms_comm();
  if (ctas > cap) ctas = cap;
  kv_push_kernel<<<(int)ctas, threads, 0, s>>>(
      reinterpret_cast<const uint8_t*>(src_k), reinterpret_cast<const uint8_t*>(src_v),
      reinterpret_cast<uint8_t*>(dst_k), reinterpret_cast<uint8_t*>(dst_v), pairs, n_pairs, src_heads, dst_heads,
      src_h0, dst_h0, n_heads, chunk_bytes, src_blocks, dst_blocks, ready, status,
      reinterpret_cast<unsigned long long*>(span));
  return (int)ctas;
}

// ------------------------------------------------------------- segments
// segs: [n, 3] int64 of (src address, dst address, bytes); addresses and
// sizes must be 16-byte aligned.  Each warp walks one segment at a time.
__global__ void __launch_bounds__(256) copy_segments_kernel(const int64_t* __restrict__ segs, int n,
                                                            uint32_t* ready, int* status) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int gw = blockIdx.x * wpb + (threadIdx.x >> 5);
  const int nw = gridDim.x * wpb;
  for (int s = 0; s < n; ++s) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(segs[3 * s]);
    uint8_t* dst = reinterpret_cast<uint8_t*>(segs[3 * s + 1]);
    const int64_t bytes = segs[3 * s + 2];
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | (uintptr_t)bytes) & 15) != 0) {
      record_status(status, CX_ERR_BOUNDS);
      continue;
    }
    const int64_t nv = bytes >> 4;
    // 4 vectors per lane per step: a warp moves 2 KB per iteration
    int64_t i = ((int64_t)gw * 32 + lane);
    const int64_t stride = (int64_t)nw * 32;
    for (; i + 3 * stride < nv; i += 4 * stride) {
      u128 r0 = ld_nc_v4(src + i * 16), r1 = ld_nc_v4(src + (i + stride) * 16);
      u128 r2 = ld_nc_v4(src + (i + 2 * stride) * 16), r3 = ld_nc_v4(src + (i + 3 * stride) * 16);
      st_cs_v4(dst + i * 16, r0);
      st_cs_v4(dst + (i + stride) * 16, r1);
      st_cs_v4(dst + (i + 2 * stride) * 16, r2);
      st_cs_v4(dst + (i + 3 * stride) * 16, r3);
    }
    for (; i < nv; i += stride) st_cs_v4(dst + i * 16, ld_nc_v4(src + i * 16));
  }
  signal_done(ready);
}

int copy_segments(const int64_t* segs, int n, int64_t total_bytes, uint32_t* ready, int max_ctas, int* status,
                  cudaStream_t s) {
  if (n <= 0) return 0;
  long ctas = (long)((total_bytes + 65535) / 65536);
  if (ctas < 1) ctas = 1;
  const long cap = max_ctas > 0 ? max_ctas : 2L * num_sms_comm();
  if (ctas > cap) ctas = cap;
  copy_segments_kernel<<<(int)ctas, 256, 0, s>>>(segs, n, ready, status);
  return (int)ctas;
}

// ---------------------------------------------------------------- flags
__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status) {
  if (threadIdx.x == 0) wait_flag_geq(flag, target, timeout_ns, status);
}
__global__ void write_flag_kernel(uint32_t* flag, uint32_t value, int add) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (add)
      red_release_sys_add_u32(flag, value);
    else
      st_release_sys_u32(flag, value);
  }
}

void wait_flag(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status, cudaStream_t s) {
  wait_flag_kernel<<<1, 32, 0, s>>>(flag, target, timeout_ns, status);
}
void write_flag(uint32_t* flag, uint32_t value, bool add, cudaStream_t s) {
  write_flag_kernel<<<1, 32, 0, s>>>(flag, value, add ? 1 : 0);
}

int num_sms_comm() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

}  // namespace cx

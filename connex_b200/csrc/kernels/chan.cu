// GPU-driven point-to-point channel kernel (one launch per side per message).
//
// Copies up to CH_MAX_SEGS (src, dst, bytes) segments -- 16-byte aligned, one
// side of each being another GPU's memory mapped through CUDA IPC -- after a
// bounded wait on a u32 counter, then signals the other side:
//   mode 1 (sender): every CTA adds 1 (release, system scope) to the
//          receiver's `ready` counter once its share has landed;
//   mode 2 (receiver): the last CTA to finish stores `value` (release,
//          system scope) into the sender's `credit` counter, returning the
//          ring slot.
// A wait that runs out records CX_ERR_TIMEOUT in `status`, copies nothing
// and signals nothing.  `abort` (optional) is a word in pinned host memory
// that the host raises when the peer is declared dead: a launch that sees it
// (before or while waiting) records CX_ERR_PEER and returns at once, touching
// neither the peer's memory nor its counters.
#include "common.cuh"
#include "comm.h"

namespace cx {

struct ChanSegs {
  uint64_t src[CH_MAX_SEGS];
  uint64_t dst[CH_MAX_SEGS];
  uint64_t bytes[CH_MAX_SEGS];
  int n;
};

// Bounded wait on `flag` that also gives up when the host raised `abort`.
__device__ bool wait_or_abort(const uint32_t* flag, uint32_t target, const uint32_t* abort, uint64_t limit_ns,
                              int* status) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (flag == nullptr || counter_reached(ld_acquire_sys_u32(flag), target)) return true;
    if ((it & 15u) == 0u) {
      if (abort != nullptr && ld_acquire_sys_u32(abort) != 0u) {
        record_status(status, CX_ERR_PEER);
        return false;
      }
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > limit_ns) {
        record_status(status, CX_ERR_TIMEOUT);
        return false;
      }
    }
    __nanosleep(64);
  }
}

__global__ void __launch_bounds__(256) chan_copy_kernel(ChanSegs segs, const uint32_t* wait_on, uint32_t wait_target,
                                                        uint64_t timeout_ns, const uint32_t* abort, uint32_t* signal,
                                                        uint32_t value, int mode, uint32_t* done_ctr, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (abort != nullptr && ld_acquire_sys_u32(abort) != 0u) {  // the peer is gone: leave its memory alone
      record_status(status, CX_ERR_PEER);
      ok = 0;
    } else {
      ok = (int)wait_or_abort(wait_on, wait_target, abort, timeout_ns, status);
    }
  }
  __syncthreads();
  if (!ok) return;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5) * 32;
  for (int s = 0; s < segs.n; ++s) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(segs.src[s]);
    uint8_t* dst = reinterpret_cast<uint8_t*>(segs.dst[s]);
    const int64_t nv = (int64_t)(segs.bytes[s] >> 4);
    int64_t i = (int64_t)gw * 32 + lane;
    for (; i + 3 * stride < nv; i += 4 * stride) {
      const u128 a = ld_nc_v4(src + i * 16), b = ld_nc_v4(src + (i + stride) * 16);
      const u128 c = ld_nc_v4(src + (i + 2 * stride) * 16), d = ld_nc_v4(src + (i + 3 * stride) * 16);
      st_v4(dst + i * 16, a);
      st_v4(dst + (i + stride) * 16, b);
      st_v4(dst + (i + 2 * stride) * 16, c);
      st_v4(dst + (i + 3 * stride) * 16, d);
    }
    for (; i < nv; i += stride) st_v4(dst + i * 16, ld_nc_v4(src + i * 16));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (mode == 1) {
      red_release_sys_add_u32(signal, 1u);
    } else if (mode == 2) {
      const uint32_t prev = atomicAdd(done_ctr, 1u);
      if (prev == gridDim.x - 1) {      // every CTA's copy is done
        *done_ctr = 0;
        __threadfence_system();
        st_release_sys_u32(signal, value);
      }
    }
  }
}

void chan_copy(const uint64_t* src, const uint64_t* dst, const uint64_t* bytes, int n, const uint32_t* wait_on,
               uint32_t wait_target, uint64_t timeout_ns, const uint32_t* abort, uint32_t* signal, uint32_t value,
               int mode, uint32_t* done_ctr, int ctas, int* status, cudaStream_t s) {
  if (n < 0 || n > CH_MAX_SEGS) throw std::runtime_error("cx chan: 0..8 segments per launch");
  ChanSegs c{};
  for (int i = 0; i < n; ++i) {
    if ((src[i] | dst[i] | bytes[i]) & 15) throw std::runtime_error("cx chan: segments must be 16-byte aligned");
    c.src[i] = src[i];
    c.dst[i] = dst[i];
    c.bytes[i] = bytes[i];
  }
  c.n = n;
  if (mode == 2 && done_ctr == nullptr) throw std::runtime_error("cx chan: receiver mode needs a CTA counter");
  chan_copy_kernel<<<ctas < 1 ? 1 : ctas, 256, 0, s>>>(c, wait_on, wait_target, timeout_ns, abort, signal, value,
                                                       mode, done_ctr, status);
}

}  // namespace cx

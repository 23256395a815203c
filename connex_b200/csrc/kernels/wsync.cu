// RL weight-sync kernel: one pass that reads the trainer's weights (fp32
// master or bf16, trainer layout), casts to bf16, re-lays them out into the
// serving engine's fused layout (q|k|v rows concatenated, gate/up rows
// interleaved in blocks) and stores them
//   * through an NVLink multicast address (multimem.st: NVSwitch replicates
//     every 16-byte store to all GPUs bound to the multicast object, so the
//     trainer's egress is the model size once, whatever the receiver count),
//   * or to each of up to WS_MAX_DST destination bases with plain stores
//     (peer-push fallback, or a local fused cast+re-layout copy when the
//     source is another GPU's buffer mapped through CUDA IPC),
//   * or, scattered, each 16 bytes to ONE destination chosen by its arena
//     offset (destination p owns [p * scatter_bytes, (p + 1) * scatter_bytes)):
//     the first half of a scatter + all-gather broadcast, whose sender
//     egress is the model size once without multicast.
// When every CTA is done it releases (system scope) +1 on the receivers'
// flag words -- through the multicast address, or on each destination -- so a
// receiver's stream waits on that flag instead of a host barrier.
//
// Job table (int64 [n_jobs, WS_JOB_COLS]):
//   src, dst_off(bytes), rows, cols, src_ld, dst_ld, blk, blk_stride, blk_off,
//   src_fp32, task0, rows_per_task
// Row r of a job lands on destination row (r / blk) * blk_stride + r % blk + blk_off.
#include <algorithm>

#include "common.cuh"
#include "comm.h"

namespace cx {
namespace {

constexpr int WS_THREADS = 256;
constexpr int WS_UNROLL = 4;

struct WsDst {
  uint64_t base[WS_MAX_DST];
  uint64_t flag[WS_MAX_DST];
  int n;
  uint64_t mc_base;  // nonzero: multicast destination (base[] unused)
  uint64_t mc_flag;
  int64_t scatter;   // nonzero: each store goes to base[offset / scatter] only
};

__device__ __forceinline__ void multimem_st_v4(uint64_t addr, const u128& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void multimem_red_release_add(uint64_t addr, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ u128 load8(const int64_t* job, int64_t r, int64_t c) {
  const int64_t src = job[0], ld = job[4];
  if (job[9]) {  // fp32 -> bf16
    const float* p = reinterpret_cast<const float*>(src) + r * ld + c;
    const u128 a = ld_nc_v4(p), b = ld_nc_v4(p + 4);
    u128 o;
    o.x = pack_bf16x2(__uint_as_float(a.x), __uint_as_float(a.y));
    o.y = pack_bf16x2(__uint_as_float(a.z), __uint_as_float(a.w));
    o.z = pack_bf16x2(__uint_as_float(b.x), __uint_as_float(b.y));
    o.w = pack_bf16x2(__uint_as_float(b.z), __uint_as_float(b.w));
    return o;
  }
  return ld_nc_v4(reinterpret_cast<const uint16_t*>(src) + r * ld + c);
}

__global__ void __launch_bounds__(WS_THREADS) wsync_kernel(const int64_t* __restrict__ jobs, int n_jobs,
                                                           int64_t n_tasks, WsDst dst) {
  __shared__ int64_t job[WS_JOB_COLS];
  for (int64_t task = blockIdx.x; task < n_tasks; task += gridDim.x) {
    if (threadIdx.x == 0) {
      int lo = 0, hi = n_jobs - 1;  // last job with task0 <= task
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (jobs[(int64_t)mid * WS_JOB_COLS + 10] <= task) lo = mid; else hi = mid - 1;
      }
      for (int k = 0; k < WS_JOB_COLS; ++k) job[k] = jobs[(int64_t)lo * WS_JOB_COLS + k];
    }
    __syncthreads();
    const int64_t rows = job[2], cols = job[3], rpt = job[11];
    const int64_t r0 = (task - job[10]) * rpt;
    const int64_t nr = min(rpt, rows - r0);
    const int64_t cpr = cols >> 3;  // 16-byte output chunks per row
    const int64_t total = nr * cpr;
    const int64_t blk = job[6], bstride = job[7], boff = job[8], dld = job[5], doff = job[1];
    for (int64_t i0 = threadIdx.x; i0 < total; i0 += (int64_t)WS_THREADS * WS_UNROLL) {
      u128 v[WS_UNROLL];
      int64_t d[WS_UNROLL];
#pragma unroll
      for (int u = 0; u < WS_UNROLL; ++u) {
        const int64_t i = i0 + (int64_t)u * WS_THREADS;
        if (i < total) {
          const int64_t r = r0 + i / cpr, c = (i % cpr) << 3;
          v[u] = load8(job, r, c);
          const int64_t drow = (r / blk) * bstride + (r % blk) + boff;
          d[u] = doff + (drow * dld + c) * 2;
        }
      }
#pragma unroll
      for (int u = 0; u < WS_UNROLL; ++u) {
        if (i0 + (int64_t)u * WS_THREADS < total) {
          if (dst.mc_base) {
            multimem_st_v4(dst.mc_base + d[u], v[u]);
          } else if (dst.scatter) {
            const int64_t q = d[u] / dst.scatter;
            const int p = q < dst.n - 1 ? (int)q : dst.n - 1;
            st_v4(reinterpret_cast<void*>(dst.base[p] + d[u]), v[u]);
          } else {
            for (int p = 0; p < dst.n; ++p) st_v4(reinterpret_cast<void*>(dst.base[p] + d[u]), v[u]);
          }
        }
      }
    }
    __syncthreads();  // job[] is rewritten by the next task
  }
  __syncthreads();
  if (dst.mc_flag) {
    if (threadIdx.x == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      multimem_red_release_add(dst.mc_flag, 1u);
    }
  } else if (threadIdx.x < dst.n && dst.flag[threadIdx.x]) {
    // one release per destination, each from its own thread (in parallel)
    red_release_sys_add_u32(reinterpret_cast<uint32_t*>(dst.flag[threadIdx.x]), 1u);
  }
}

}  // namespace

int wsync(const int64_t* jobs_dev, const int64_t* jobs_host, int n_jobs, int64_t dst_bytes, const uint64_t* dst_bases,
          const uint64_t* dst_flags, int n_dst, uint64_t mc_base, uint64_t mc_flag, int max_ctas, int64_t scatter_bytes,
          cudaStream_t s) {
  if (n_jobs <= 0) return 0;
  if (!mc_base && (n_dst <= 0 || n_dst > WS_MAX_DST)) throw std::runtime_error("cx wsync: bad destination count");
  if (mc_base % 16) throw std::runtime_error("cx wsync: multicast base not 16-byte aligned");
  if (scatter_bytes < 0 || scatter_bytes % 16 || (scatter_bytes && mc_base))
    throw std::runtime_error("cx wsync: scatter size must be a multiple of 16 bytes, without multicast");
  int64_t n_tasks = 0;
  for (int j = 0; j < n_jobs; ++j) {
    const int64_t* q = jobs_host + (int64_t)j * WS_JOB_COLS;
    const int64_t src = q[0], doff = q[1], rows = q[2], cols = q[3], sld = q[4], dld = q[5], blk = q[6],
                  bstride = q[7], boff = q[8], f32 = q[9], task0 = q[10], rpt = q[11];
    const int64_t esz = f32 ? 4 : 2;
    if (rows <= 0 || cols <= 0 || cols % 8 || sld < cols || dld < cols || blk <= 0 || rpt <= 0 || boff < 0 ||
        bstride < 0)
      throw std::runtime_error("cx wsync: bad job shape");
    if (src % 16 || (sld * esz) % 16 || doff % 16 || (dld * 2) % 16)
      throw std::runtime_error("cx wsync: job not 16-byte aligned");
    if (task0 != n_tasks) throw std::runtime_error("cx wsync: task0 column not a running prefix");
    // the last destination row written: the largest row index of the last block
    int64_t max_row = 0;
    const int64_t last = rows - 1;
    max_row = (last / blk) * bstride + (last % blk) + boff;
    if (rows > blk) max_row = std::max(max_row, (last / blk - 1) * bstride + (blk - 1) + boff);
    if (doff + (max_row * dld + cols) * 2 > dst_bytes) throw std::runtime_error("cx wsync: job past destination");
    n_tasks += (rows + rpt - 1) / rpt;
  }
  WsDst d{};
  d.n = mc_base ? 0 : n_dst;
  for (int p = 0; p < d.n; ++p) {
    if (dst_bases[p] % 16) throw std::runtime_error("cx wsync: destination base not 16-byte aligned");
    d.base[p] = dst_bases[p];
    d.flag[p] = dst_flags ? dst_flags[p] : 0;
  }
  d.mc_base = mc_base;
  d.mc_flag = mc_flag;
  d.scatter = scatter_bytes;
  const int sms = num_sms_comm();
  int ctas = (int)std::min<int64_t>(n_tasks, (int64_t)sms * 4);
  if (max_ctas > 0) ctas = std::min(ctas, max_ctas);
  wsync_kernel<<<ctas, WS_THREADS, 0, s>>>(jobs_dev, n_jobs, n_tasks, d);
  return ctas;
}

}  // namespace cx

// Expert-parallel MoE layer over NVLink peer memory, fused with the expert
// GEMMs (see moe.h for the kernel sequence).
//
// Layout of the receive side of rank d: rows of local slot s occupy
// [seg(s), seg(s+1)); inside a slot, rows are ordered by source rank, so a
// sender computes every destination offset from the all-gathered count
// matrix counts[src][dst][slot] without a round trip.  Each routed row also
// carries (source rank, t*K+k, routing weight) so the down-projection GEMM
// can store its weighted output row straight into the source's combine
// buffer.  Every cross-rank wait is a bounded acquire on a u32 counter.
#include <algorithm>
#include <stdexcept>

#include "common.cuh"
#include "gemm.h"
#include "moe.h"

namespace cx {

// Self-check of a vector access: a pointer that is not 16-byte aligned is
// recorded as status 100 + site and the access is skipped (never faults).
__device__ __forceinline__ bool aligned16(const void* p, int site, int* status) {
  if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) return true;
  record_status(status, 100 + site);
  return false;
}

// ------------------------------------------------------------------ count
__global__ void __launch_bounds__(1024) ep_count_kernel(const int* __restrict__ topk_idx, const int* __restrict__ l2p,
                                                        const int* __restrict__ l2p_cnt, int max_rep, int T, int K,
                                                        int N, int S, int me, int* __restrict__ pos,
                                                        int* __restrict__ slot_of, EpPeers peers, uint32_t* comb_expect,
                                                        uint32_t arrivals_per_row, int* status) {
  extern __shared__ int hist[];  // [N*S]
  __shared__ int valid;
  const int NB = N * S;
  for (int i = threadIdx.x; i < NB; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x == 0) valid = 0;
  __syncthreads();
  int my_valid = 0;
  const int TK = T * K;
  const int lane = threadIdx.x & 31;
  constexpr int U = 4;  // routed rows per thread per pass: their dependent loads overlap
  for (int base = 0; base < TK; base += blockDim.x * U) {  // uniform trip count: whole warps take part
    int idx[U], e[U], c[U], slot[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      idx[u] = base + u * blockDim.x + threadIdx.x;
      e[u] = idx[u] < TK ? topk_idx[idx[u]] : -1;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) c[u] = e[u] >= 0 ? l2p_cnt[e[u]] : 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      // spread a token's replicas by token index
      slot[u] = c[u] > 0 ? l2p[e[u] * max_rep + ((idx[u] / K) % c[u])] : -1;
      if (slot[u] >= NB) slot[u] = -1;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      // one shared-memory atomic per distinct slot in the warp (skewed routing hits few slots)
      const unsigned grp = __match_any_sync(0xffffffffu, slot[u]);
      const int leader = __ffs(grp) - 1;
      int b = 0;
      if (slot[u] >= 0 && lane == leader) b = atomicAdd(&hist[slot[u]], __popc(grp));
      b = __shfl_sync(0xffffffffu, b, leader);
      if (idx[u] < TK) {
        if (slot[u] < 0) {
          slot_of[idx[u]] = -1;
          pos[idx[u]] = -1;
        } else {
          slot_of[idx[u]] = slot[u];
          pos[idx[u]] = b + __popc(grp & ((1u << lane) - 1u));
          ++my_valid;
        }
      }
    }
  }
  atomicAdd(&valid, my_valid);
  __syncthreads();
  for (int d = 0; d < N; ++d) {
    int* cm = reinterpret_cast<int*>(peers.counts[d]);
    for (int i = threadIdx.x; i < NB; i += blockDim.x) cm[me * NB + i] = hist[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(comb_expect, (uint32_t)valid * arrivals_per_row);
  // one release per destination, each from its own thread: they run in
  // parallel (a release from one thread to N flags would be N system fences
  // in a row); the barrier above makes every thread's peer stores part of
  // what each release publishes
  if (threadIdx.x < N) red_release_sys_add_u32(reinterpret_cast<uint32_t*>(peers.count_flag[threadIdx.x]), 1u);
}

// --------------------------------------------------------------- dispatch
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const float* __restrict__ topk_w,
                                                          const int* __restrict__ pos, const int* __restrict__ slot_of,
                                                          const int* counts, int T, int K, int H, int N, int S, int me,
                                                          int R_max, uint32_t count_target, EpPeers peers,
                                                          int* status) {
  extern __shared__ int off[];  // [N*S]: first row of (me -> dst, slot) at dst; then tot[N*S]
  __shared__ int ok;
  if (threadIdx.x == 0)
    ok = wait_flag_geq(reinterpret_cast<const uint32_t*>(peers.count_flag[me]), count_target, kDefaultWaitNs, status);
  __syncthreads();
  if (!ok) return;
  const int NB = N * S;
  int* tot = off + NB;  // rows of (dst, slot) from every source
  // one pass over the count matrix, every thread on its own (dst, slot): N loads each, in parallel
  for (int i = threadIdx.x; i < NB; i += blockDim.x) {
    const int d = i / S, s = i - d * S;
    int all = 0, before_me = 0;
    for (int src = 0; src < N; ++src) {
      const int c = (int)ld_acquire_gpu_u32((const uint32_t*)&counts[(src * N + d) * S + s]);
      all += c;
      if (src < me) before_me += c;
    }
    tot[i] = all;
    off[i] = before_me;
  }
  __syncthreads();
  // slot s of dst d starts after every source's rows of slots < s (prefix from shared memory)
  for (int i = threadIdx.x; i < NB; i += blockDim.x) {
    const int d = i / S, s = i - d * S;
    int base = 0;
    for (int s2 = 0; s2 < s; ++s2) base += tot[d * S + s2];
    off[i] += base;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int nvec = H / 8;  // 16-byte vectors per row
  const int TK = T * K;
  const int n_warps = gridDim.x * wpb;
  // each warp takes `chunk` consecutive routed rows at a time (up to 32, fewer when there are
  // few rows, so every warp has work): their slot / position / weight are loaded once
  // (coalesced) and broadcast, so no row waits on its own metadata loads
  const int chunk = max(1, min(32, (TK + n_warps - 1) / n_warps));
  for (int c0 = (blockIdx.x * wpb + (threadIdx.x >> 5)) * chunk; c0 < TK; c0 += n_warps * chunk) {
    int my_slot = -1, my_pos = 0;
    float my_w = 0.f;
    if (lane < chunk && c0 + lane < TK) {
      my_slot = slot_of[c0 + lane];
      my_pos = pos[c0 + lane];
      my_w = topk_w[c0 + lane];
    }
    const int n_rows = min(chunk, TK - c0);
    for (int j = 0; j < n_rows; ++j) {
      const int i = c0 + j;
      const int slot = __shfl_sync(0xffffffffu, my_slot, j);
      const int p = __shfl_sync(0xffffffffu, my_pos, j);
      const float wt = __shfl_sync(0xffffffffu, my_w, j);
      if (slot < 0) continue;
      const int d = slot / S;
      const int row = off[slot] + p;
      if (row < 0 || row >= R_max) {
        record_status(status, CX_ERR_BOUNDS);
        continue;
      }
      const u128* src = reinterpret_cast<const u128*>(x + (size_t)(i / K) * H);
      u128* dst = reinterpret_cast<u128*>(reinterpret_cast<__nv_bfloat16*>(peers.recv[d]) + (size_t)row * H);
      if (!aligned16(src, 1, status) || !aligned16(dst, 1, status)) continue;
      // 8 loads per lane in flight before the stores (a 2048-wide bf16 row is exactly 256 vectors)
      constexpr int ILP = 8;
      int v0 = 0;
      for (; v0 + 32 * ILP <= nvec; v0 += 32 * ILP) {
        u128 buf[ILP];
#pragma unroll
        for (int q = 0; q < ILP; ++q) buf[q] = ld_nc_v4(src + v0 + lane + 32 * q);
#pragma unroll
        for (int q = 0; q < ILP; ++q) st_cs_v4(dst + v0 + lane + 32 * q, buf[q]);
      }
      for (int v = v0 + lane; v < nvec; v += 32) st_cs_v4(dst + v, ld_nc_v4(src + v));
      if (lane == 0) {
        int4 m = make_int4(me, i, __float_as_int(wt), 0);
        int4* mp = reinterpret_cast<int4*>(peers.recv_meta[d]) + row;
        if (aligned16(mp, 2, status)) *mp = m;
      }
    }
  }
  __syncthreads();
  // the rows are stored: one release per destination, in parallel threads
  if (threadIdx.x < N) red_release_sys_add_u32(reinterpret_cast<uint32_t*>(peers.data_flag[threadIdx.x]), 1u);
}

// ------------------------------------------------------- grouped GEMM
namespace epg {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192, MAXS = 256;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256 + (MAXS + 1) * 4 * 2;
}  // namespace epg

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

__global__ void __launch_bounds__(epg::THREADS, 1)
    ep_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           int n_per_expert, int K, __nv_bfloat16* __restrict__ D, int ldd, const int* counts, int N,
                           int S, int me, int mode, const int4* __restrict__ meta, EpPeers peers, int H,
                           const uint32_t* wait_flag, uint32_t wait_target, int R_max, int* status) {
  using namespace epg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* seg = reinterpret_cast<int*>(smem + STAGES * STAGE_BYTES + 256);  // [S+1] row starts
  int* tpre = seg + (MAXS + 1);                                          // [S+1] tile prefix
  __shared__ int ok;
  __shared__ unsigned comb_rows[EP_MAX_RANKS];  // mode 1: rows stored into each source's combine buffer
  for (int i = threadIdx.x; i < EP_MAX_RANKS; i += blockDim.x) comb_rows[i] = 0u;

  const int warp = warp_id(), lane = lane_id();
  const int n_tiles = n_per_expert / BN;
  if (threadIdx.x == 0) ok = wait_flag == nullptr ? 1 : (int)wait_flag_geq(wait_flag, wait_target, kDefaultWaitNs, status);
  __syncthreads();
  if (ok) {  // rows per local expert, summed over sources by all threads in parallel
    for (int e = threadIdx.x; e < S; e += blockDim.x) {
      int rows = 0;
      for (int src = 0; src < N; ++src) rows += ld_acquire_gpu_u32((const uint32_t*)&counts[(src * N + me) * S + e]);
      tpre[e] = rows;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && ok) {  // prefixes (in place): row starts and tile starts
    int r = 0, t = 0;
    for (int e = 0; e < S; ++e) {
      const int rows = tpre[e];
      seg[e] = r;
      tpre[e] = t;
      r += rows;
      t += ((rows + BM - 1) / BM) * n_tiles;
    }
    seg[S] = r;
    tpre[S] = t;
    if (r > R_max) {  // counts beyond the receive capacity: do nothing, report
      record_status(status, CX_ERR_BOUNDS);
      ok = 0;
    }
  }
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
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = ok ? tpre[S] : 0;
  const int nk = (K + BK - 1) / BK;

  auto locate = [&](int t, int& e, int& mt, int& nt) {
    int lo = 0, hi = S - 1;  // last e with tpre[e] <= t (empty experts share a prefix)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tpre[mid] <= t) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int r = t - tpre[e];
    mt = r / n_tiles;
    nt = r - mt * n_tiles;
  };

  if (warp == 0) {
    if (lane == 0) {
      fence_proxy_async_global();  // peer stores acquired above -> visible to TMA
      bool good = true;
      uint32_t stage = 0, phase = 0;
      for (int t = blockIdx.x; t < total && good; t += gridDim.x) {
        int e, mt, nt;
        locate(t, e, mt, nt);
        const int arow = seg[e] + mt * BM;
        const int brow = e * n_per_expert + nt * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status)) {
            good = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, arow);
          tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, brow);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool good = true, issued = false;
      for (int t = blockIdx.x; t < total && good; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, status)) {
          good = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, status)) {
            good = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES), b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), IDESC, (kb | k) ? 1u : 0u);
          issued = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!good) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (!acc) acc_phase ^= 1;
      }
      if (!good && issued) {
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr, 100000000ull);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    uint32_t acc = 0, acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int e, mt, nt;
      locate(t, e, mt, nt);
      if (!mbar_wait(&tfull[acc], acc_phase, status)) break;
      tc_fence_after();
      const int local_row = mt * BM + q * 32 + lane;
      const bool valid = local_row < seg[e + 1] - seg[e];
      const int row = seg[e] + local_row;
      const uint32_t tb = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if (mode == 0) {
        constexpr int HALF = BN / 2;
#pragma unroll 1
        for (int c = 0; c < HALF / 32; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(tb + c * 32, g);
          tmem_ld32(tb + HALF + c * 32, u);
          tmem_ld_wait();
          if (valid) {
            u128 out[4];
            uint32_t* o = reinterpret_cast<uint32_t*>(out);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              o[j] = pack_bf16x2(silu_f(__uint_as_float(g[2 * j])) * __uint_as_float(u[2 * j]),
                                 silu_f(__uint_as_float(g[2 * j + 1])) * __uint_as_float(u[2 * j + 1]));
            __nv_bfloat16* dst = D + (size_t)row * ldd + nt * HALF + c * 32;
            if (aligned16(dst, 3, status)) {
#pragma unroll
              for (int v = 0; v < 4; ++v) st_v4(dst + v * 8, out[v]);
            }
          }
        }
      } else {
        int4 m = make_int4(-1, 0, 0, 0);
        if (valid && aligned16(meta + row, 4, status)) m = meta[row];
        const int src = m.x, tk = m.y;
        const float w = __int_as_float(m.z);
        const bool ok_src = valid && src >= 0 && src < N;
        __nv_bfloat16* dst = ok_src ? reinterpret_cast<__nv_bfloat16*>(peers.comb[src]) + (size_t)tk * H + nt * BN
                                    : nullptr;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tb + c * 32, r);
          tmem_ld_wait();
          if (ok_src && aligned16(dst + c * 32, 5, status)) {
            u128 out[4];
            uint32_t* o = reinterpret_cast<uint32_t*>(out);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              o[j] = pack_bf16x2(__uint_as_float(r[2 * j]) * w, __uint_as_float(r[2 * j + 1]) * w);
#pragma unroll
            for (int v = 0; v < 4; ++v) st_cs_v4(dst + c * 32 + v * 8, out[v]);
          }
        }
        if (valid && !ok_src) record_status(status, CX_ERR_BOUNDS);
        // count this tile's rows per source; the CTA releases them once, after its last tile
        const int key = ok_src ? src : -1;
        const unsigned peers_mask = __match_any_sync(0xffffffffu, key);
        if (key >= 0 && lane == __ffs(peers_mask) - 1) atomicAdd(&comb_rows[key], (unsigned)__popc(peers_mask));
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (!acc) acc_phase ^= 1;
    }
    if (mode != 0) __threadfence_system();  // this thread's combine stores, before the CTA's releases
  }
  __syncthreads();
  if (mode != 0 && threadIdx.x < N && comb_rows[threadIdx.x])
    red_release_sys_add_u32(reinterpret_cast<uint32_t*>(peers.comb_flag[threadIdx.x]), comb_rows[threadIdx.x]);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ----------------------------------------------------------------- combine
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* __restrict__ comb,
                                                         const int* __restrict__ slot_of, int T, int K, int H,
                                                         __nv_bfloat16* __restrict__ y, const uint32_t* comb_flag,
                                                         const uint32_t* expect, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flag_geq(comb_flag, ld_acquire_gpu_u32(expect), kDefaultWaitNs, status);
  __syncthreads();
  if (!ok) return;
  const int nvec = H / 8;
  for (long idx = (long)blockIdx.x * blockDim.x + threadIdx.x; idx < (long)T * nvec; idx += (long)gridDim.x * blockDim.x) {
    const int t = (int)(idx / nvec), v = (int)(idx - (long)t * nvec);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < K; ++k) {
      if (slot_of[t * K + k] < 0) continue;
      const __nv_bfloat16* cp = comb + ((size_t)(t * K + k) * H) + v * 8;
      if (!aligned16(cp, 6, status)) continue;
      u128 r = ld_v4(cp);
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += bf16_lo(p[j]);
        acc[2 * j + 1] += bf16_hi(p[j]);
      }
    }
    u128 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    if (aligned16(y + (size_t)t * H + v * 8, 7, status)) st_v4(y + (size_t)t * H + v * 8, o);
  }
}

// ------------------------------------------------------------------- host
void ep_count(const int* topk_idx, const int* l2p, const int* l2p_cnt, int max_rep, int T, int K, int N, int S,
              int me, int* pos, int* slot_of, EpPeers peers, uint32_t* comb_expect, int arrivals_per_row, int* status,
              cudaStream_t s) {
  ep_count_kernel<<<1, 1024, N * S * sizeof(int), s>>>(topk_idx, l2p, l2p_cnt, max_rep, T, K, N, S, me, pos, slot_of,
                                                         peers, comb_expect, (uint32_t)arrivals_per_row, status);
}

void ep_dispatch(const void* x, const float* topk_w, const int* pos, const int* slot_of, const int* counts_local,
                 int T, int K, int H, int N, int S, int me, int R_max, uint32_t count_target, EpPeers peers,
                 int* status, cudaStream_t s) {
  if (H % 8) throw std::runtime_error("cx ep_dispatch: hidden size must be a multiple of 8");
  if (2L * N * S * sizeof(int) > 48 * 1024) throw std::runtime_error("cx ep_dispatch: too many (rank, slot) pairs");
  ep_dispatch_kernel<<<EP_DISPATCH_CTAS, 256, 2 * N * S * sizeof(int), s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), topk_w, pos, slot_of, counts_local, T, K, H, N, S, me, R_max,
      count_target, peers, status);
}

// Small per-thread cache of 128-byte-swizzled bf16 tensor maps, keyed by
// everything the map encodes (base, extents, stride, box).
static CUtensorMap cached_tmap(const void* base, uint64_t inner, uint64_t outer, uint64_t stride, uint32_t box_in,
                               uint32_t box_out) {
  struct Entry {
    const void* base;
    uint64_t inner, outer, stride;
    uint32_t box_in, box_out;
    CUtensorMap map;
  };
  constexpr int CAP = 16;
  thread_local Entry cache[CAP];
  thread_local int used = 0, next = 0;
  for (int i = 0; i < used; ++i) {
    const Entry& e = cache[i];
    if (e.base == base && e.inner == inner && e.outer == outer && e.stride == stride && e.box_in == box_in &&
        e.box_out == box_out)
      return e.map;
  }
  Entry& e = cache[next];
  e = Entry{base, inner, outer, stride, box_in, box_out, make_tmap_bf16_2d(base, inner, outer, stride, box_in, box_out, true)};
  next = (next + 1) % CAP;
  if (used < CAP) ++used;
  return e.map;
}

void ep_grouped_gemm(const void* A, int lda, const void* B, int n_per_expert, int K, void* D, int ldd,
                     const int* counts_local, int N, int S, int me, int R_max, int mode, const int* recv_meta,
                     EpPeers peers, int H, const uint32_t* wait_flag, uint32_t wait_target, int* status,
                     cudaStream_t s) {
  using namespace epg;
  if (S > MAXS) throw std::runtime_error("cx ep gemm: too many local experts");
  if (N > EP_MAX_RANKS) throw std::runtime_error("cx ep gemm: too many EP ranks");
  if (n_per_expert % BN || K % 8) throw std::runtime_error("cx ep gemm: expert width must be a multiple of 256");
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(ep_grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    attr[dev & 63] = true;
  }
  // The operands of a layer's two GEMMs (receive / mid buffers, expert
  // weights) stay put between forwards: their tensor maps are encoded once.
  const CUtensorMap ta = cached_tmap(A, (uint64_t)K, (uint64_t)R_max, (uint64_t)lda * 2, BK, BM);
  const CUtensorMap tb = cached_tmap(B, (uint64_t)K, (uint64_t)S * n_per_expert, (uint64_t)K * 2, BK, BN);
  ep_grouped_gemm_kernel<<<num_sms(), THREADS, SMEM, s>>>(ta, tb, n_per_expert, K,
                                                          reinterpret_cast<__nv_bfloat16*>(D), ldd, counts_local, N, S,
                                                          me, mode, reinterpret_cast<const int4*>(recv_meta), peers, H,
                                                          wait_flag, wait_target, R_max, status);
}

void ep_combine(const void* comb, const int* slot_of, int T, int K, int H, void* y, const uint32_t* comb_flag,
                const uint32_t* expect, int* status, cudaStream_t s) {
  if (T == 0) return;
  long work = (long)T * (H / 8);
  int ctas = (int)std::min<long>((work + 255) / 256, 4L * num_sms());
  ep_combine_kernel<<<ctas, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(comb), slot_of, T, K, H,
                                         reinterpret_cast<__nv_bfloat16*>(y), comb_flag, expect, status);
}

}  // namespace cx

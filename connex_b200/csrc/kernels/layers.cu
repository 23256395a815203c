// Memory-bound transformer-layer kernels of the serving runtime:
//   * rmsnorm / fused residual-add + rmsnorm (one CTA per token row),
//   * rope + paged-KV write: rotates q and k of the fused QKV projection in
//     place (rotate-half convention, fp32 cos/sin cache) and writes the
//     rotated k and v of every token straight into its paged-cache slot,
//   * embedding gather, greedy argmax over the vocabulary.
// All I/O is 16-byte vectorised; the fp32 math mirrors the torch reference.
#include "common.cuh"
#include "layers.h"

namespace cx {

// ---------------------------------------------------------------- RMSNorm
// x: [T, H] bf16 (ld ldx).  residual (optional): [T, H], updated in place to
// x + residual before the norm.  out: [T, H] = norm(.) * w.
template <int VPT>  // 16-byte vectors per thread
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                      __nv_bfloat16* residual, int ldr,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ out, int ldo, int H, float eps) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  float v[VPT * 8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + tid) * 8;
    if (c < H) {
      u128 a = ld_v4(x + (size_t)row * ldx + c);
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      if (residual != nullptr) {
        u128 r = ld_v4(residual + (size_t)row * ldr + c);
        const uint32_t* pr = reinterpret_cast<const uint32_t*>(&r);
        u128 s;
        uint32_t* ps = reinterpret_cast<uint32_t*>(&s);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // round the sum to bf16 first: the residual stream is stored in bf16
          ps[j] = pack_bf16x2(bf16_lo(pa[j]) + bf16_lo(pr[j]), bf16_hi(pa[j]) + bf16_hi(pr[j]));
          v[i * 8 + 2 * j] = bf16_lo(ps[j]);
          v[i * 8 + 2 * j + 1] = bf16_hi(ps[j]);
        }
        st_v4(residual + (size_t)row * ldr + c, s);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[i * 8 + 2 * j] = bf16_lo(pa[j]);
          v[i * 8 + 2 * j + 1] = bf16_hi(pa[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i * 8 + j] * v[i * 8 + j];
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float t = tid < (blockDim.x >> 5) ? red[tid] : 0.f;
    t = warp_sum(t);
    if (tid == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * blockDim.x + tid) * 8;
    if (c < H) {
      u128 wv = ld_v4(w + c);
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
      u128 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        po[j] = pack_bf16x2(v[i * 8 + 2 * j] * inv * bf16_lo(pw[j]), v[i * 8 + 2 * j + 1] * inv * bf16_hi(pw[j]));
      st_v4(out + (size_t)row * ldo + c, o);
    }
  }
}

void rmsnorm(const void* x, int ldx, void* residual, int ldr, const void* w, void* out, int ldo, int T, int H,
             float eps, cudaStream_t s) {
  if (T == 0) return;
  const int threads = 256;
  const int vpt = (H / 8 + threads - 1) / threads;
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto R = reinterpret_cast<__nv_bfloat16*>(residual);
  auto W = reinterpret_cast<const __nv_bfloat16*>(w);
  auto O = reinterpret_cast<__nv_bfloat16*>(out);
  if (vpt <= 1)
    rmsnorm_kernel<1><<<T, threads, 0, s>>>(X, ldx, R, ldr, W, O, ldo, H, eps);
  else if (vpt <= 2)
    rmsnorm_kernel<2><<<T, threads, 0, s>>>(X, ldx, R, ldr, W, O, ldo, H, eps);
  else if (vpt <= 4)
    rmsnorm_kernel<4><<<T, threads, 0, s>>>(X, ldx, R, ldr, W, O, ldo, H, eps);
  else
    rmsnorm_kernel<8><<<T, threads, 0, s>>>(X, ldx, R, ldr, W, O, ldo, H, eps);
}

// ------------------------------------------------------- RoPE + cache write
// qkv: [T, (Hq + 2*Hkv) * D] bf16 (ld ldq), rotated in place for q and k.
// cos_sin: [max_pos, D] fp32, cos in [0, D/2), sin in [D/2, D).
// slot_mapping: [T] int64 (-1 = do not cache).  Caches: [blocks, Hkv, BS, D].
// One warp per (token, head); D = 128 -> 4 elements per lane.
// Optional per-head RMSNorm of q and k before the rotation (``qn`` / ``kn``:
// [D] bf16 weights, Qwen3-style query/key norm), fused into the same pass.
__global__ void rope_cache_kernel(__nv_bfloat16* qkv, int ldq, const int* __restrict__ pos,
                                  const float* __restrict__ cos_sin, const int64_t* __restrict__ slots,
                                  __nv_bfloat16* kc, __nv_bfloat16* vc, int T, int Hq, int Hkv, int BS,
                                  int num_blocks, int max_pos, int* status, const __nv_bfloat16* __restrict__ qn,
                                  const __nv_bfloat16* __restrict__ kn, float eps) {
  constexpr int D = 128;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  if (gw >= T * heads) return;
  const int t = gw / heads;
  const int h = gw - t * heads;
  __nv_bfloat16* row = qkv + (size_t)t * ldq + (size_t)h * D;
  // lane owns elements {2*lane, 2*lane+1} of the first half and their partners
  const int i = lane * 2;  // 0..62
  uint32_t lo = *reinterpret_cast<const uint32_t*>(row + i);
  uint32_t hi = *reinterpret_cast<const uint32_t*>(row + i + D / 2);
  if (h < Hq + Hkv) {
    const int p = pos[t];
    if (p < 0 || p >= max_pos) {
      record_status(status, CX_ERR_BOUNDS);
      return;
    }
    const float* cs = cos_sin + (size_t)p * D;
    const float c0 = cs[i], c1 = cs[i + 1], s0 = cs[D / 2 + i], s1 = cs[D / 2 + i + 1];
    float x0 = bf16_lo(lo), x1 = bf16_hi(lo), y0 = bf16_lo(hi), y1 = bf16_hi(hi);
    const __nv_bfloat16* nw = h < Hq ? qn : kn;
    if (nw != nullptr) {
      const float ss = warp_sum(x0 * x0 + x1 * x1 + y0 * y0 + y1 * y1);
      const float r = rsqrtf(ss * (1.0f / D) + eps);
      const uint32_t wl = *reinterpret_cast<const uint32_t*>(nw + i);
      const uint32_t wh = *reinterpret_cast<const uint32_t*>(nw + i + D / 2);
      // round to bf16 between the norm and the rotation, like a separate norm layer
      x0 = __bfloat162float(__float2bfloat16(x0 * r * bf16_lo(wl)));
      x1 = __bfloat162float(__float2bfloat16(x1 * r * bf16_hi(wl)));
      y0 = __bfloat162float(__float2bfloat16(y0 * r * bf16_lo(wh)));
      y1 = __bfloat162float(__float2bfloat16(y1 * r * bf16_hi(wh)));
    }
    lo = pack_bf16x2(x0 * c0 - y0 * s0, x1 * c1 - y1 * s1);
    hi = pack_bf16x2(y0 * c0 + x0 * s0, y1 * c1 + x1 * s1);
    *reinterpret_cast<uint32_t*>(row + i) = lo;
    *reinterpret_cast<uint32_t*>(row + i + D / 2) = hi;
  }
  if (h >= Hq && slots != nullptr) {
    const int64_t slot = slots[t];
    if (slot < 0) return;
    const int64_t blk = slot / BS;
    const int off = (int)(slot - blk * BS);
    if (blk >= num_blocks) {
      record_status(status, CX_ERR_BOUNDS);
      return;
    }
    const bool is_k = h < Hq + Hkv;
    const int kvh = is_k ? h - Hq : h - Hq - Hkv;
    __nv_bfloat16* dst = (is_k ? kc : vc) + (((size_t)blk * Hkv + kvh) * BS + off) * D;
    *reinterpret_cast<uint32_t*>(dst + i) = lo;
    *reinterpret_cast<uint32_t*>(dst + i + D / 2) = hi;
  }
}

void rope_cache(void* qkv, int ldq, const int* pos, const float* cos_sin, const int64_t* slots, void* kc, void* vc,
                int T, int Hq, int Hkv, int D, int BS, int num_blocks, int max_pos, int* status, cudaStream_t s,
                const void* q_norm, const void* k_norm, float eps) {
  if (T == 0) return;
  if (D != 128) throw std::runtime_error("cx rope: head_dim must be 128");
  const long warps = (long)T * (Hq + 2 * Hkv);
  const int threads = 256;
  const long blocks = (warps * 32 + threads - 1) / threads;
  rope_cache_kernel<<<blocks, threads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(qkv), ldq, pos, cos_sin, slots,
                                               reinterpret_cast<__nv_bfloat16*>(kc),
                                               reinterpret_cast<__nv_bfloat16*>(vc), T, Hq, Hkv, BS, num_blocks,
                                               max_pos, status, reinterpret_cast<const __nv_bfloat16*>(q_norm),
                                               reinterpret_cast<const __nv_bfloat16*>(k_norm), eps);
}

// --------------------------------------------------------------- embedding
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int H, int V, int* status) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= V) {
    record_status(status, CX_ERR_BOUNDS);
    id = 0;
  }
  const u128* src = reinterpret_cast<const u128*>(table + (size_t)id * H);
  u128* dst = reinterpret_cast<u128*>(out + (size_t)t * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

void embedding(const int* ids, const void* table, void* out, int T, int H, int V, int* status, cudaStream_t s) {
  if (T == 0) return;
  embedding_kernel<<<T, 256, 0, s>>>(ids, reinterpret_cast<const __nv_bfloat16*>(table),
                                     reinterpret_cast<__nv_bfloat16*>(out), H, V, status);
}

// ------------------------------------------------------------------ argmax
// logits: [B, V] bf16 (ld ldl) -> out[B] int32.  Ties resolve to the lowest index.
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16* __restrict__ logits, int ldl, int V,
                                                      int* __restrict__ out) {
  const int b = blockIdx.x;
  const __nv_bfloat16* row = logits + (size_t)b * ldl;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    u128 v = ld_nc_v4(row + c * 8);
    const uint32_t* p = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = bf16_lo(p[j]), bb = bf16_hi(p[j]);
      int ia = c * 8 + 2 * j;
      if (a > best || (a == best && ia < bi)) { best = a; bi = ia; }
      if (bb > best || (bb == best && ia + 1 < bi)) { best = bb; bi = ia + 1; }
    }
  }
  for (int c = nvec * 8 + threadIdx.x; c < V; c += blockDim.x) {
    float a = __bfloat162float(row[c]);
    if (a > best || (a == best && c < bi)) { best = a; bi = c; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ob = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) { sb[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sb[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ob = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (threadIdx.x == 0) out[b] = bi;
  }
}

void argmax(const void* logits, int ldl, int B, int V, int* out, cudaStream_t s) {
  if (B == 0) return;
  argmax_kernel<<<B, 1024, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(logits), ldl, V, out);
}

// ---------------------------------------------------------------- row gather
// out[i, :] = src[idx[i], :] for bf16 rows of H elements (H % 8 == 0).
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, int lds, const int* __restrict__ idx,
                                   __nv_bfloat16* __restrict__ out, int ldo, int H) {
  const int i = blockIdx.x;
  const u128* s = reinterpret_cast<const u128*>(src + (size_t)idx[i] * lds);
  u128* d = reinterpret_cast<u128*>(out + (size_t)i * ldo);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) d[c] = s[c];
}

void gather_rows(const void* src, int lds, const int* idx, void* out, int ldo, int n, int H, cudaStream_t s) {
  if (n == 0) return;
  gather_rows_kernel<<<n, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(src), lds, idx,
                                       reinterpret_cast<__nv_bfloat16*>(out), ldo, H);
}

}  // namespace cx

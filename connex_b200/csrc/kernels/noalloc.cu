// Allocation-free decode attention entry point (declared in noalloc.h).
//
// The split-K partial results live in a file-scope device array instead of a
// caller workspace.  Host code never passes the array's name to a kernel (in
// host code that name is only a host-side stand-in): the device address is
// looked up once per device with cudaGetSymbolAddress while that device is
// current, checked, cached, and handed to the existing decode kernels.
#include <mutex>
#include <stdexcept>

#include "layers.h"
#include "noalloc.h"

namespace {

__device__ __align__(256) float g_decode_scratch[CX_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of this device's scratch; resolved on the first call.
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CX_NOALLOC_ERR_SYMBOL;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return CX_NOALLOC_ERR_SYMBOL;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return CX_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) size_t cx_decode_attention_noalloc_scratch_floats(int B, int Hq,
                                                                                                    int max_ctx) {
  if (B <= 0 || Hq <= 0 || max_ctx <= 0) return 0;
  return (size_t)B * (size_t)Hq * (size_t)cx::decode_attention_splits(max_ctx) * 130u;
}

extern "C" __attribute__((visibility("default"))) const char* cx_noalloc_error_string(int code) {
  switch (code) {
    case CX_NOALLOC_OK: return "ok";
    case CX_NOALLOC_ERR_TOO_LARGE:
      return "decode attention needs more scratch than the built-in CX_NOALLOC_SCRATCH_FLOATS; "
             "use fewer sequences or a shorter max context per call";
    case CX_NOALLOC_ERR_SYMBOL: return "could not resolve the device address of the built-in scratch";
    case CX_NOALLOC_ERR_ARGS: return "unsupported arguments (GQA group must be 1, 2, 4 or 8; sizes must be > 0)";
    case CX_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
    default: return "unknown error";
  }
}

extern "C" __attribute__((visibility("default"))) int cx_decode_attention_noalloc(
    const void* q, int ldq, const void* k_cache, const void* v_cache, const int* block_tables, int max_blocks,
    const int* ctx_lens, void* out, int ldo, int B, int Hq, int Hkv, int BS, int max_ctx, float scale,
    cudaStream_t stream) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || BS <= 0 || max_ctx <= 0 || Hq % Hkv != 0) return CX_NOALLOC_ERR_ARGS;
  const int G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return CX_NOALLOC_ERR_ARGS;
  if (cx_decode_attention_noalloc_scratch_floats(B, Hq, max_ctx) > (size_t)CX_NOALLOC_SCRATCH_FLOATS)
    return CX_NOALLOC_ERR_TOO_LARGE;
  float* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != CX_NOALLOC_OK) return rc;
  try {
    // The whole array is this call's workspace, so small batches get the
    // finer split plan (more CTAs) the allocating path uses when its
    // workspace has room; the plan never asks for more than it is given.
    cx::decode_attention(q, ldq, k_cache, v_cache, block_tables, max_blocks, ctx_lens, out, ldo, B, Hq, Hkv, BS,
                         max_ctx, scale, scratch, stream, (long)CX_NOALLOC_SCRATCH_FLOATS);
  } catch (const std::exception&) {
    return CX_NOALLOC_ERR_ARGS;
  }
  if (cudaPeekAtLastError() != cudaSuccess) {
    (void)cudaGetLastError();
    return CX_NOALLOC_ERR_LAUNCH;
  }
  return CX_NOALLOC_OK;
}

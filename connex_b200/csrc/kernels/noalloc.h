// Allocation-free C entry point of the paged decode attention.
//
// This entry point has no counterpart in the reference (HeterInfra/connex
// ships no kernels at all); it is an addition of this library.
//
// Who it is for: callers that cannot call cudaMalloc.  A serving engine
// typically reserves nearly all of a GPU's memory up front for its KV cache
// and weights, so a late cudaMalloc fails or must evict; and C callers that
// link this library directly, without PyTorch's caching allocator, cannot
// afford cudaMalloc / cudaFree on the decode path because both can
// synchronize the device.  Such callers pass inputs and outputs they already
// own; the split-K scratch of the attention lives in a fixed device array
// inside this library instead of a caller-provided workspace.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

// Capacity of the built-in scratch, in floats (4 MiB per GPU that loads the
// library, held until the process exits).  A call needs
// B * Hq * ceil(max_ctx / 512) * 130 floats.
#define CX_NOALLOC_SCRATCH_FLOATS (1u << 20)

enum {
  CX_NOALLOC_OK = 0,
  CX_NOALLOC_ERR_TOO_LARGE = -1,   // the call needs more scratch than CX_NOALLOC_SCRATCH_FLOATS
  CX_NOALLOC_ERR_SYMBOL = -2,      // cudaGetSymbolAddress of the scratch failed on this device
  CX_NOALLOC_ERR_ARGS = -3,        // unsupported shape (GQA group not 1/2/4/8, head_dim != 128, ...)
  CX_NOALLOC_ERR_LAUNCH = -4,      // the kernel launch reported an error
};

// Same operation and arguments as the allocating entry point
// (connex_b200._C.decode_attention), minus the workspace:
//   q            [B, ldq] bf16, q heads first (head h at column h*128)
//   k/v cache    [blocks, Hkv, BS, 128] bf16
//   block_tables [B, max_blocks] int32, ctx_lens [B] int32 (tokens incl. the new one)
//   out          [B, ldo] bf16 (Hq*128 columns written)
// Launches on `stream` and returns CX_NOALLOC_OK or an error code; never
// allocates or frees device or host memory.
//
// The first call on a device resolves the device address of the scratch
// (cudaGetSymbolAddress, with that device current); make that first call
// before any stream capture.  Every call on a device shares the one scratch
// array and leaves its contents behind; calls whose kernels overlap on the
// GPU (different streams, no ordering between them) race on it and must be
// serialized by the caller.  No part of the scratch needs to start at zero:
// every slot a call reads is written earlier in the same call.
int cx_decode_attention_noalloc(const void* q, int ldq, const void* k_cache, const void* v_cache,
                                const int* block_tables, int max_blocks, const int* ctx_lens, void* out,
                                int ldo, int B, int Hq, int Hkv, int BS, int max_ctx, float scale,
                                cudaStream_t stream);

// Scratch floats a call with these sizes needs (compare with CX_NOALLOC_SCRATCH_FLOATS).
size_t cx_decode_attention_noalloc_scratch_floats(int B, int Hq, int max_ctx);

// Human-readable text of an error code.
const char* cx_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif

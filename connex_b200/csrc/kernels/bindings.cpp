// pybind11 bindings of the connex_b200._C extension (sm_100a kernels plus
// CUDA IPC plumbing for peer buffers).  Every op launches on the current
// torch stream of the tensor's device and never allocates device memory
// itself: outputs and workspaces come from the caller.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "comm.h"
#include "gemm.h"
#include "layers.h"
#include "moe.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")

cudaStream_t cur_stream(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

int* status_ptr(const c10::optional<at::Tensor>& st) {
  if (!st.has_value()) return nullptr;
  TORCH_CHECK(st->scalar_type() == at::kInt && st->is_cuda(), "status must be an int32 CUDA tensor");
  return st->data_ptr<int>();
}

int row_ld(const at::Tensor& t) {
  TORCH_CHECK(t.dim() == 2, "expected a 2-D tensor");
  TORCH_CHECK(t.stride(1) == 1, "rows must be contiguous");
  return (int)t.stride(0);
}

// D = A . B^T (+ R) | SiLU-mul epilogue.  A [M,K], B [N,K], D [M,N or N/2].
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& R, int64_t epi,
          int64_t bn, const c10::optional<at::Tensor>& status, int64_t max_ctas,
          const c10::optional<at::Tensor>& workspace, int64_t splits) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  CHECK_CUDA(D);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_BF16(D);
  const c10::cuda::CUDAGuard g(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1), N = (int)B.size(0);
  TORCH_CHECK(B.size(1) == K, "gemm: K mismatch");
  if (epi == cx::EPI_SILU_MUL) {
    TORCH_CHECK(D.size(0) == M && D.size(1) == N / 2, "gemm: SiLU-mul output must be [M, N/2]");
  } else {
    TORCH_CHECK(D.size(0) == M && D.size(1) == N, "gemm: output shape mismatch");
  }
  const void* rp = nullptr;
  int ldr = 0;
  if (epi == cx::EPI_ADD) {
    TORCH_CHECK(R.has_value(), "gemm: residual epilogue needs R");
    CHECK_BF16((*R));
    rp = R->data_ptr();
    ldr = row_ld(*R);
  }
  if (M == 0) return;
  float* W = nullptr;
  if (splits > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->is_cuda() && workspace->scalar_type() == at::kFloat &&
                    workspace->is_contiguous() && workspace->numel() >= (int64_t)M * N,
                "gemm: split-K needs a contiguous fp32 CUDA workspace of at least M*N elements (kept zero)");
    W = workspace->data_ptr<float>();
  }
  cx::gemm_bf16_tn(A.data_ptr(), B.data_ptr(), D.data_ptr(), rp, M, N, K, row_ld(A), row_ld(B), row_ld(D), ldr,
                   (int)epi, (int)bn, status_ptr(status), (int)max_ctas, cur_stream(A), W, (int)splits);
}

int64_t gemm_splits(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t bn) {
  return cx::gemm_splits((int)M, (int)N, (int)K, (int)epi, (int)bn);
}

void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& out,
             double eps) {
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(out);
  const c10::cuda::CUDAGuard g(x.device());
  void* rp = nullptr;
  int ldr = 0;
  if (residual.has_value()) {
    rp = residual->data_ptr();
    ldr = row_ld(*residual);
  }
  const int H = (int)x.size(1);
  TORCH_CHECK(H % 8 == 0, "rmsnorm: hidden size must be a multiple of 8");
  cx::rmsnorm(x.data_ptr(), row_ld(x), rp, ldr, w.data_ptr(), out.data_ptr(), row_ld(out), (int)x.size(0), H,
              (float)eps, cur_stream(x));
}

void rope_cache(at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& cos_sin,
                const c10::optional<at::Tensor>& slots, const c10::optional<at::Tensor>& kc,
                const c10::optional<at::Tensor>& vc, int64_t Hq, int64_t Hkv, const c10::optional<at::Tensor>& status,
                const c10::optional<at::Tensor>& q_norm, const c10::optional<at::Tensor>& k_norm, double eps) {
  CHECK_BF16(qkv);
  const void* qn = nullptr;
  const void* kn = nullptr;
  for (const auto* w : {&q_norm, &k_norm})
    if (w->has_value())
      TORCH_CHECK((*w)->is_cuda() && (*w)->scalar_type() == at::kBFloat16 && (*w)->numel() == 128 &&
                      (*w)->is_contiguous(),
                  "rope_cache: q/k norm weights must be contiguous bf16 CUDA [128]");
  if (q_norm.has_value()) qn = q_norm->data_ptr();
  if (k_norm.has_value()) kn = k_norm->data_ptr();
  TORCH_CHECK(pos.scalar_type() == at::kInt, "positions must be int32");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat, "cos_sin must be fp32");
  const c10::cuda::CUDAGuard g(qkv.device());
  const int64_t* sp = nullptr;
  void *kp = nullptr, *vp = nullptr;
  int BS = 16, nb = 0;
  if (slots.has_value()) {
    TORCH_CHECK(slots->scalar_type() == at::kLong, "slot_mapping must be int64");
    TORCH_CHECK(kc.has_value() && vc.has_value(), "rope_cache: caches required with a slot mapping");
    sp = slots->data_ptr<int64_t>();
    kp = kc->data_ptr();
    vp = vc->data_ptr();
    nb = (int)kc->size(0);
    BS = (int)kc->size(2);
  }
  cx::rope_cache(qkv.data_ptr(), row_ld(qkv), pos.data_ptr<int>(), cos_sin.data_ptr<float>(), sp, kp, vp,
                 (int)qkv.size(0), (int)Hq, (int)Hkv, 128, BS, nb, (int)cos_sin.size(0), status_ptr(status),
                 cur_stream(qkv), qn, kn, (float)eps);
}

void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out,
               const c10::optional<at::Tensor>& status) {
  TORCH_CHECK(ids.scalar_type() == at::kInt, "ids must be int32");
  const c10::cuda::CUDAGuard g(table.device());
  cx::embedding(ids.data_ptr<int>(), table.data_ptr(), out.data_ptr(), (int)ids.numel(), (int)table.size(1),
                (int)table.size(0), status_ptr(status), cur_stream(table));
}

void argmax(const at::Tensor& logits, at::Tensor& out) {
  CHECK_BF16(logits);
  TORCH_CHECK(out.scalar_type() == at::kInt, "argmax output must be int32");
  const c10::cuda::CUDAGuard g(logits.device());
  cx::argmax(logits.data_ptr(), row_ld(logits), (int)logits.size(0), (int)logits.size(1), out.data_ptr<int>(),
             cur_stream(logits));
}

void gather_rows(const at::Tensor& src, const at::Tensor& idx, at::Tensor& out) {
  const c10::cuda::CUDAGuard g(src.device());
  cx::gather_rows(src.data_ptr(), row_ld(src), idx.data_ptr<int>(), out.data_ptr(), row_ld(out), (int)idx.numel(),
                  (int)src.size(1), cur_stream(src));
}

void prefill_attention_tc(const at::Tensor& qkv, at::Tensor& out, const at::Tensor& tile_info, int64_t Hq,
                          int64_t Hkv, double scale, const c10::optional<at::Tensor>& status, int64_t tile_rows) {
  CHECK_BF16(qkv);
  CHECK_BF16(out);
  TORCH_CHECK(tile_rows == 128 || tile_rows == 256, "tile_rows must be 128 or 256");
  TORCH_CHECK(tile_info.scalar_type() == at::kInt && tile_info.dim() == 2 && tile_info.size(1) == 3,
              "tile_info must be int32 [n, 3]");
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * 128, "qkv must hold exactly (Hq + 2 Hkv) heads of 128");
  const c10::cuda::CUDAGuard g(qkv.device());
  cx::prefill_attention_tc(qkv.data_ptr(), row_ld(qkv), (int)qkv.size(1), (int)qkv.size(0), out.data_ptr(),
                           row_ld(out), tile_info.data_ptr<int>(), (int)tile_info.size(0), (int)Hq, (int)Hkv,
                           (float)scale, status_ptr(status), cur_stream(qkv), (int)tile_rows);
}

void prefill_attention_paged(const at::Tensor& qkv, const at::Tensor& kc, const at::Tensor& vc,
                             const at::Tensor& block_tables, at::Tensor& out, const at::Tensor& tile_info, int64_t Hq,
                             int64_t Hkv, double scale, const c10::optional<at::Tensor>& status,
                             int64_t tile_rows) {
  TORCH_CHECK(tile_rows == 128 || tile_rows == 256, "tile_rows must be 128 or 256");
  CHECK_BF16(qkv);
  CHECK_BF16(kc);
  CHECK_BF16(vc);
  CHECK_BF16(out);
  TORCH_CHECK(tile_info.scalar_type() == at::kInt && tile_info.dim() == 2 && tile_info.size(1) == 5,
              "tile_info must be int32 [n, 5]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.is_contiguous(),
              "block_tables must be contiguous int32 [B, max_blocks]");
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * 128, "qkv must hold exactly (Hq + 2 Hkv) heads of 128");
  TORCH_CHECK(kc.dim() == 4 && kc.size(1) == Hkv && kc.size(2) == 16 && kc.size(3) == 128 && kc.is_contiguous() &&
                  vc.is_contiguous() && vc.sizes() == kc.sizes(),
              "caches must be contiguous [blocks, Hkv, 16, 128]");
  const c10::cuda::CUDAGuard g(qkv.device());
  cx::prefill_attention_paged_tc(qkv.data_ptr(), row_ld(qkv), (int)qkv.size(1), (int)qkv.size(0), kc.data_ptr(),
                                 vc.data_ptr(), kc.size(0) * Hkv * 16, block_tables.data_ptr<int>(),
                                 (int)block_tables.size(1), out.data_ptr(), row_ld(out), tile_info.data_ptr<int>(),
                                 (int)tile_info.size(0), (int)Hq, (int)Hkv, (float)scale, status_ptr(status),
                                 cur_stream(qkv), (int)tile_rows);
}

void decode_attention(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& block_tables,
                      const at::Tensor& ctx_lens, at::Tensor& out, int64_t Hq, int64_t max_ctx, double scale,
                      at::Tensor& workspace) {
  CHECK_BF16(q);
  CHECK_BF16(kc);
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt, "int32 tables");
  TORCH_CHECK(workspace.scalar_type() == at::kFloat, "workspace must be fp32");
  const c10::cuda::CUDAGuard g(q.device());
  const int B = (int)q.size(0);
  const int Hkv = (int)kc.size(1), BS = (int)kc.size(2);
  TORCH_CHECK(kc.dim() == 4 && kc.size(3) == 128 && kc.is_contiguous() && vc.is_contiguous() && vc.sizes() == kc.sizes(),
              "caches must be contiguous [blocks, Hkv, BS, 128]");
  const int splits = cx::decode_attention_splits((int)max_ctx);
  TORCH_CHECK(workspace.numel() >= (int64_t)B * Hq * splits * 130, "decode workspace too small");
  cx::decode_attention(q.data_ptr(), row_ld(q), kc.data_ptr(), vc.data_ptr(), block_tables.data_ptr<int>(),
                       (int)block_tables.size(1), ctx_lens.data_ptr<int>(), out.data_ptr(), row_ld(out), B, (int)Hq,
                       Hkv, BS, (int)max_ctx, (float)scale, workspace.data_ptr<float>(), cur_stream(q),
                       (long)workspace.numel(), nullptr, (long)kc.size(0));
}

int64_t decode_attention_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t max_ctx, int64_t ws_floats) {
  return cx::decode_attention_plan((int)B, (int)Hq, (int)Hkv, (int)max_ctx, (long)ws_floats);
}

int64_t decode_workspace_floats(int64_t B, int64_t Hq, int64_t max_ctx) {
  return B * Hq * cx::decode_attention_splits((int)max_ctx) * 130;
}

// ---- peer-memory movement (addresses may be local or peer-mapped) ----------
int64_t kv_push_layer(int64_t src_k, int64_t src_v, int64_t dst_k, int64_t dst_v, const at::Tensor& pairs,
                      int64_t src_heads, int64_t dst_heads, int64_t src_h0, int64_t dst_h0, int64_t n_heads,
                      int64_t chunk_bytes, int64_t src_blocks, int64_t dst_blocks, int64_t ready, int64_t max_ctas,
                      const c10::optional<at::Tensor>& status, int64_t span, int64_t threads) {
  TORCH_CHECK(pairs.scalar_type() == at::kInt && pairs.is_cuda(), "pairs must be int32 CUDA [n, 2]");
  const c10::cuda::CUDAGuard g(pairs.device());
  return cx::kv_push_layer(reinterpret_cast<const void*>(src_k), reinterpret_cast<const void*>(src_v),
                           reinterpret_cast<void*>(dst_k), reinterpret_cast<void*>(dst_v), pairs.data_ptr<int>(),
                           (int)pairs.size(0), (int)src_heads, (int)dst_heads, (int)src_h0, (int)dst_h0, (int)n_heads,
                           (int)chunk_bytes, (int)src_blocks, (int)dst_blocks, reinterpret_cast<uint32_t*>(ready),
                           (int)max_ctas, status_ptr(status), cur_stream(pairs), reinterpret_cast<uint64_t*>(span),
                           (int)threads);
}

int64_t copy_segments(const at::Tensor& segs, int64_t total_bytes, int64_t ready, int64_t max_ctas,
                      const c10::optional<at::Tensor>& status) {
  TORCH_CHECK(segs.scalar_type() == at::kLong && segs.is_cuda() && segs.dim() == 2 && segs.size(1) == 3,
              "segs must be int64 CUDA [n, 3]");
  const c10::cuda::CUDAGuard g(segs.device());
  return cx::copy_segments(segs.data_ptr<int64_t>(), (int)segs.size(0), total_bytes,
                           reinterpret_cast<uint32_t*>(ready), (int)max_ctas, status_ptr(status), cur_stream(segs));
}

// Weight sync: jobs int64 [n, WS_JOB_COLS] on the device and its host copy
// (validated here); destinations are a multicast address or up to
// WS_MAX_DST plain bases (with optional flag words).
int64_t wsync(const at::Tensor& jobs_dev, const at::Tensor& jobs_cpu, int64_t dst_bytes, std::vector<int64_t> bases,
              std::vector<int64_t> flags, int64_t mc_base, int64_t mc_flag, int64_t max_ctas, int64_t scatter_bytes) {
  TORCH_CHECK(jobs_dev.is_cuda() && jobs_dev.scalar_type() == at::kLong && jobs_dev.is_contiguous() &&
                  jobs_dev.dim() == 2 && jobs_dev.size(1) == cx::WS_JOB_COLS,
              "jobs_dev must be contiguous int64 CUDA [n, ", cx::WS_JOB_COLS, "]");
  TORCH_CHECK(!jobs_cpu.is_cuda() && jobs_cpu.scalar_type() == at::kLong && jobs_cpu.is_contiguous() &&
                  jobs_cpu.sizes() == jobs_dev.sizes(),
              "jobs_cpu must be the contiguous host copy of jobs_dev");
  TORCH_CHECK(flags.empty() || flags.size() == bases.size(), "one flag per destination (or none)");
  const c10::cuda::CUDAGuard g(jobs_dev.device());
  return cx::wsync(jobs_dev.data_ptr<int64_t>(), jobs_cpu.data_ptr<int64_t>(), (int)jobs_dev.size(0), dst_bytes,
                   reinterpret_cast<const uint64_t*>(bases.data()),
                   flags.empty() ? nullptr : reinterpret_cast<const uint64_t*>(flags.data()), (int)bases.size(),
                   (uint64_t)mc_base, (uint64_t)mc_flag, (int)max_ctas, scatter_bytes, cur_stream(jobs_dev));
}

void chan_copy(std::vector<int64_t> src, std::vector<int64_t> dst, std::vector<int64_t> bytes, int64_t wait_on,
               int64_t wait_target, int64_t timeout_ns, int64_t signal, int64_t value, int64_t mode, int64_t done_ctr,
               int64_t ctas, const at::Tensor& status, int64_t abort) {
  TORCH_CHECK(src.size() == dst.size() && dst.size() == bytes.size(), "chan_copy: segment lists differ in length");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "chan_copy: status must be an int32 CUDA word");
  const c10::cuda::CUDAGuard g(status.device());
  cx::chan_copy(reinterpret_cast<const uint64_t*>(src.data()), reinterpret_cast<const uint64_t*>(dst.data()),
                reinterpret_cast<const uint64_t*>(bytes.data()), (int)src.size(),
                reinterpret_cast<const uint32_t*>(wait_on), (uint32_t)wait_target, (uint64_t)timeout_ns,
                reinterpret_cast<const uint32_t*>(abort), reinterpret_cast<uint32_t*>(signal), (uint32_t)value,
                (int)mode, reinterpret_cast<uint32_t*>(done_ctr), (int)ctas, status.data_ptr<int>(), cur_stream(status));
}

void wait_flag(int64_t flag, int64_t target, int64_t timeout_ns, const at::Tensor& status) {
  const c10::cuda::CUDAGuard g(status.device());
  cx::wait_flag(reinterpret_cast<const uint32_t*>(flag), (uint32_t)target, (uint64_t)timeout_ns,
                status.data_ptr<int>(), cur_stream(status));
}

void write_flag(int64_t flag, int64_t value, bool add, const at::Tensor& like) {
  const c10::cuda::CUDAGuard g(like.device());
  cx::write_flag(reinterpret_cast<uint32_t*>(flag), (uint32_t)value, add, cur_stream(like));
}

// ---- expert parallelism -------------------------------------------------------
// peers: int64 CUDA tensor [7, N] of addresses (counts, count_flag, recv,
// recv_meta, data_flag, comb, comb_flag) on every rank.
cx::EpPeers ep_peers(const at::Tensor& peers) {
  TORCH_CHECK(peers.scalar_type() == at::kLong && peers.is_cuda() && peers.dim() == 2 && peers.size(0) == 7,
              "peers must be int64 CUDA [7, N]");
  const uint64_t* p = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  const int64_t N = peers.size(1);
  return cx::EpPeers{p, p + N, p + 2 * N, p + 3 * N, p + 4 * N, p + 5 * N, p + 6 * N};
}

void ep_count(const at::Tensor& topk_idx, const at::Tensor& l2p, const at::Tensor& l2p_cnt, int64_t S, int64_t me,
              at::Tensor& pos, at::Tensor& slot_of, const at::Tensor& peers, at::Tensor& comb_expect,
              int64_t arrivals_per_row, const c10::optional<at::Tensor>& status) {
  const c10::cuda::CUDAGuard g(topk_idx.device());
  TORCH_CHECK(topk_idx.scalar_type() == at::kInt && topk_idx.is_contiguous() && topk_idx.dim() == 2,
              "topk_idx must be contiguous int32 [T, K]");
  TORCH_CHECK(pos.numel() >= topk_idx.numel() && slot_of.numel() >= topk_idx.numel(),
              "ep_count: pos / slot_of hold fewer than T*K entries (more tokens than the layer's capacity)");
  TORCH_CHECK(l2p.scalar_type() == at::kInt && l2p.dim() == 2 && l2p_cnt.numel() == l2p.size(0),
              "l2p must be int32 [E, R] with l2p_cnt [E]");
  cx::ep_count(topk_idx.data_ptr<int>(), l2p.data_ptr<int>(), l2p_cnt.data_ptr<int>(), (int)l2p.size(1),
               (int)topk_idx.size(0), (int)topk_idx.size(1), (int)peers.size(1), (int)S, (int)me, pos.data_ptr<int>(),
               slot_of.data_ptr<int>(), ep_peers(peers), reinterpret_cast<uint32_t*>(comb_expect.data_ptr<int>()),
               (int)arrivals_per_row, status_ptr(status), cur_stream(topk_idx));
}

void ep_dispatch(const at::Tensor& x, const at::Tensor& topk_w, const at::Tensor& pos, const at::Tensor& slot_of,
                 const at::Tensor& counts_local, int64_t K, int64_t S, int64_t me, int64_t R_max, int64_t count_target,
                 const at::Tensor& peers, const c10::optional<at::Tensor>& status) {
  CHECK_BF16(x);
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.is_contiguous() && topk_w.is_contiguous() && topk_w.numel() == x.size(0) * K,
              "ep_dispatch: x [T, H] and topk_w [T, K] must be contiguous and agree");
  TORCH_CHECK(pos.numel() >= x.size(0) * K, "ep_dispatch: more tokens than the layer's capacity");
  cx::ep_dispatch(x.data_ptr(), topk_w.data_ptr<float>(), pos.data_ptr<int>(), slot_of.data_ptr<int>(),
                  counts_local.data_ptr<int>(), (int)x.size(0), (int)K, (int)x.size(1), (int)peers.size(1), (int)S,
                  (int)me, (int)R_max, (uint32_t)count_target, ep_peers(peers), status_ptr(status), cur_stream(x));
}

void ep_grouped_gemm(const at::Tensor& A, const at::Tensor& B, int64_t n_per_expert, at::Tensor& D,
                     const at::Tensor& counts_local, int64_t S, int64_t me, int64_t mode, const at::Tensor& recv_meta,
                     const at::Tensor& peers, int64_t H, int64_t wait_flag, int64_t wait_target,
                     const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(B);
  const c10::cuda::CUDAGuard g(A.device());
  cx::ep_grouped_gemm(A.data_ptr(), row_ld(A), B.data_ptr(), (int)n_per_expert, (int)A.size(1), D.data_ptr(),
                      (int)D.stride(0), counts_local.data_ptr<int>(), (int)peers.size(1), (int)S, (int)me,
                      (int)A.size(0), (int)mode, recv_meta.data_ptr<int>(), ep_peers(peers), (int)H,
                      reinterpret_cast<const uint32_t*>(wait_flag), (uint32_t)wait_target, status_ptr(status),
                      cur_stream(A));
}

void ep_combine(const at::Tensor& comb, const at::Tensor& slot_of, int64_t T, int64_t K, at::Tensor& y,
                int64_t comb_flag, const at::Tensor& expect, const c10::optional<at::Tensor>& status) {
  const c10::cuda::CUDAGuard g(comb.device());
  TORCH_CHECK(comb.size(0) >= T * K && slot_of.numel() >= T * K && y.size(0) >= T && y.size(1) == comb.size(1),
              "ep_combine: buffers smaller than T*K rows");
  cx::ep_combine(comb.data_ptr(), slot_of.data_ptr<int>(), (int)T, (int)K, (int)y.size(1), y.data_ptr(),
                 reinterpret_cast<const uint32_t*>(comb_flag), reinterpret_cast<const uint32_t*>(expect.data_ptr<int>()),
                 status_ptr(status), cur_stream(comb));
}

// The whole EP layer in one call: count, dispatch, the two grouped GEMMs and
// combine, launched back to back on the current stream (one crossing from
// Python instead of five; the kernels' own waits order the phases across
// ranks).  Targets are the cumulative u32 counter values this forward waits for.
void ep_forward(const at::Tensor& x, const at::Tensor& topk_idx, const at::Tensor& topk_w, const at::Tensor& l2p,
                const at::Tensor& l2p_cnt, at::Tensor& out, const at::Tensor& w13, const at::Tensor& w2,
                at::Tensor& pos, at::Tensor& slot_of, const at::Tensor& counts, const at::Tensor& recv,
                const at::Tensor& recv_meta, at::Tensor& mid, const at::Tensor& comb, at::Tensor& comb_expect,
                const at::Tensor& peers, int64_t S, int64_t me, int64_t ffn, int64_t R_max, int64_t count_target,
                int64_t data_flag, int64_t data_target, int64_t comb_flag, const c10::optional<at::Tensor>& status,
                const std::vector<int64_t>& events) {
  const int64_t T = x.size(0), H = x.size(1), K = topk_idx.size(1);
  TORCH_CHECK(H % 256 == 0, "ep_forward: hidden size must be a multiple of 256");
  TORCH_CHECK(events.empty() || events.size() == 6, "ep_forward: events are 6 CUDA event handles or none");
  // optional per-phase timing: events[i] recorded before phase i (and after the last)
  const cudaStream_t st = cur_stream(x);
  auto mark = [&](int i) {
    if (!events.empty()) C10_CUDA_CHECK(cudaEventRecord(reinterpret_cast<cudaEvent_t>(events[i]), st));
  };
  mark(0);
  ep_count(topk_idx, l2p, l2p_cnt, S, me, pos, slot_of, peers, comb_expect, H / 256, status);
  mark(1);
  ep_dispatch(x, topk_w, pos, slot_of, counts, K, S, me, R_max, count_target, peers, status);
  mark(2);
  ep_grouped_gemm(recv, w13, 2 * ffn, mid, counts, S, me, 0, recv_meta, peers, H, data_flag, data_target, status);
  mark(3);
  ep_grouped_gemm(mid, w2, H, mid, counts, S, me, 1, recv_meta, peers, H, data_flag, data_target, status);
  mark(4);
  ep_combine(comb, slot_of, T, K, out, comb_flag, comb_expect, status);
  mark(5);
}

// ---- CUDA IPC ---------------------------------------------------------------
// Export the allocation that contains `ptr`: returns (handle bytes, offset of
// ptr inside the allocation).
std::pair<py::bytes, int64_t> ipc_export(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  CUdeviceptr base = 0;
  size_t size = 0;
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = nullptr;
  if (range == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuMemGetAddressRange unavailable");
    range = reinterpret_cast<RangeFn>(p);
  }
  TORCH_CHECK(range(&base, &size, (CUdeviceptr)ptr) == CUDA_SUCCESS, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  return {py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)), (int64_t)(ptr - (int64_t)base)};
}

int64_t ipc_open(const std::string& handle, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

bool enable_peer_access(int64_t device, int64_t peer) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  int can = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, (int)device, (int)peer));
  if (!can) return false;
  cudaError_t e = cudaDeviceEnablePeerAccess((int)peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return true;
  }
  C10_CUDA_CHECK(e);
  return true;
}

// Wrap a raw device address as a tensor view (no ownership).
at::Tensor from_ptr(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, opts);
}

}  // namespace


PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "connex_b200 sm_100a kernels";
  m.def("gemm", &gemm, py::arg("A"), py::arg("B"), py::arg("D"), py::arg("R") = py::none(), py::arg("epi") = 0,
        py::arg("bn") = 0, py::arg("status") = py::none(), py::arg("max_ctas") = 0,
        py::arg("workspace") = py::none(), py::arg("splits") = 1);
  m.def("rmsnorm", &rmsnorm);
  m.def("rope_cache", &rope_cache, py::arg("qkv"), py::arg("pos"), py::arg("cos_sin"), py::arg("slots"),
        py::arg("kc"), py::arg("vc"), py::arg("Hq"), py::arg("Hkv"), py::arg("status") = py::none(),
        py::arg("q_norm") = py::none(), py::arg("k_norm") = py::none(), py::arg("eps") = 1e-6);
  m.def("embedding", &embedding);
  m.def("argmax", &argmax);
  m.def("gather_rows", &gather_rows);
  m.def("prefill_attention", &prefill_attention_tc);
  m.def("prefill_attention_paged", &prefill_attention_paged);
  m.def("attention_exp_split", &cx::attention_exp_split);
  m.def("attention_profile", &cx::attention_profile);
  m.def("decode_attention", &decode_attention);
  m.def("decode_attention_plan", &decode_attention_plan);
  m.def("decode_workspace_floats", &decode_workspace_floats);
  m.def("kv_push_layer", &kv_push_layer);
  m.def("gemm_splits", &gemm_splits);
  m.def("gemm_raster_group", &cx::gemm_raster_group);
  m.def("copy_segments", &copy_segments);
  m.def("wsync", &wsync, py::arg("jobs_dev"), py::arg("jobs_cpu"), py::arg("dst_bytes"), py::arg("bases"),
        py::arg("flags"), py::arg("mc_base"), py::arg("mc_flag"), py::arg("max_ctas"), py::arg("scatter_bytes") = 0);
  m.attr("WS_JOB_COLS") = cx::WS_JOB_COLS;
  m.attr("WS_MAX_DST") = cx::WS_MAX_DST;
  m.def("chan_copy", &chan_copy, py::arg("src"), py::arg("dst"), py::arg("bytes"), py::arg("wait_on"),
        py::arg("wait_target"), py::arg("timeout_ns"), py::arg("signal"), py::arg("value"), py::arg("mode"),
        py::arg("done_ctr"), py::arg("ctas"), py::arg("status"), py::arg("abort") = 0);
  m.attr("CH_MAX_SEGS") = cx::CH_MAX_SEGS;
  m.def("wait_flag", &wait_flag);
  m.def("write_flag", &write_flag);
  m.def("ep_count", &ep_count);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_grouped_gemm", &ep_grouped_gemm);
  m.def("ep_combine", &ep_combine);
  m.def("ep_forward", &ep_forward);
  m.attr("EP_DISPATCH_CTAS") = cx::EP_DISPATCH_CTAS;
  m.def("ipc_export", &ipc_export);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("enable_peer_access", &enable_peer_access);
  m.def("from_ptr", &from_ptr);
  m.attr("EPI_STORE") = (int)cx::EPI_STORE;
  m.attr("EPI_ADD") = (int)cx::EPI_ADD;
  m.attr("EPI_SILU_MUL") = (int)cx::EPI_SILU_MUL;
}

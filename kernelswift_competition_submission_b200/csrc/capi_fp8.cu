// C-ABI entry of the FP8 w8a8 expert path: quantise the token rows (per token
// per 128) -> align -> gather e4m3 rows, and their scales into a [K blocks][rows]
// table -> FP8 GEMM1 (+ SiLU*mul + per-row e4m3 quantisation of act, scales
// written as a [N blocks][rows] table) -> FP8 GEMM2 -> top-k combine.
// moe_fused_experts_fp8_rows starts from rows already quantised and packed
// (codes then scales, as the expert-parallel dispatch moves them) and can leave
// the per-slot rows in the workspace for a fused consumer.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>

namespace moe {
namespace {

inline size_t up256(size_t v) { return (v + 255) / 256 * 256; }

struct F8Layout2 {
  size_t meta, sorted, xq, xs, xq_s, xs_s, actq, acts, y, total;
  int64_t cap;
};

F8Layout2 fp8_layout(int64_t M, int E, int topk, int K, int N) {
  F8Layout2 l;
  const int64_t P = M * topk;
  l.cap = moe_align_capacity(P, E, kBlockM);
  size_t o = 0;
  l.meta = o;  o = up256(o + 4 * (size_t)align_meta_ints(E));
  l.sorted = o; o = up256(o + 4 * (size_t)l.cap);
  l.xq = o;    o = up256(o + (size_t)M * K);
  l.xs = o;    o = up256(o + 4 * (size_t)M * (K / 128));
  l.xq_s = o;  o = up256(o + (size_t)l.cap * K);
  l.xs_s = o;  o = up256(o + 4 * (size_t)l.cap * (K / 128));
  l.actq = o;  o = up256(o + (size_t)l.cap * N);
  l.acts = o;  o = up256(o + 4 * (size_t)l.cap * (N / 128));
  l.y = o;     o = up256(o + 2 * (size_t)P * K);
  l.total = o;
  return l;
}

// align -> gather e4m3 rows and their scales -> GEMM1 -> GEMM2 (-> combine when out != nullptr).
// Token t's codes at q + t * ldq (bytes), its K / 128 scales at s + t * lds (floats).
cudaError_t fp8_expert_rows(const F8Layout2& l, uint8_t* ws, const uint8_t* q, int64_t ldq, const float* s,
                            int64_t lds, const void* w1_q, const float* w1_scale, const void* w2_q,
                            const float* w2_scale, const float* topk_weights, const int32_t* topk_ids, int64_t M,
                            int E, int topk, int K, int N, bool ue8m0, void* out, int max_ctas, int* status,
                            cudaStream_t st) {
  const int64_t P = M * topk;
  const bool swap = fp8_use_swap(P, E);
  int32_t* meta = reinterpret_cast<int32_t*>(ws + l.meta);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + l.sorted);
  const AlignMeta am = align_meta_contiguous(meta, E);
  cudaError_t err = launch_align(topk_ids, P, topk, E, kBlockM, am, true, sorted, l.cap, nullptr, nullptr, 0, st);
  if (err == cudaSuccess)
    err = launch_gather_rows(q, ldq, K, sorted, am.block_start, E, topk, l.cap, ws + l.xq_s, st);
  // the block-scaled GEMMs read the row scales as UE8M0 atoms, the others as fp32
  if (err == cudaSuccess)
    err = launch_gather_scales_t(s, lds, K / 128, sorted, am.block_start, E, topk, l.cap, ue8m0 && !swap,
                                 reinterpret_cast<float*>(ws + l.xs_s), st);
  if (swap) {  // a few rows per expert: weight rows x 32-token tiles
    if (err == cudaSuccess)
      err = launch_fp8_swap_gemm1(ws + l.xq_s, reinterpret_cast<const float*>(ws + l.xs_s), l.cap, P, w1_q, w1_scale,
                                  E, K, N, am.counts, am.block_start, ws + l.actq,
                                  reinterpret_cast<float*>(ws + l.acts), ue8m0, status, max_ctas, st);
    if (err == cudaSuccess)
      err = launch_fp8_swap_gemm2(ws + l.actq, reinterpret_cast<const float*>(ws + l.acts), l.cap, P, w2_q, w2_scale,
                                  E, K, N, am.counts, am.block_start, sorted, ws + l.y, status, max_ctas, st);
  } else {
    if (err == cudaSuccess)
      err = launch_fp8_gemm1(ws + l.xq_s, reinterpret_cast<const float*>(ws + l.xs_s), l.cap, w1_q, w1_scale, E, K,
                             N, am.block_start, ws + l.actq, reinterpret_cast<float*>(ws + l.acts), ue8m0, status,
                             max_ctas, st);
    if (err == cudaSuccess)
      err = launch_fp8_gemm2(ws + l.actq, reinterpret_cast<const float*>(ws + l.acts), l.cap, w2_q, w2_scale, E, K,
                             N, am.block_start, sorted, ws + l.y, ue8m0, status, max_ctas, st);
  }
  if (err == cudaSuccess && out)
    err = launch_combine(MOE_DTYPE_BF16, ws + l.y, topk_weights, topk_ids, M, topk, E, K, out, st);
  return err;
}

inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int fp8_shape_ok(int64_t M, int E, int topk, int K, int N) {
  if (M < 0 || E <= 0 || topk <= 0 || K <= 0 || N <= 0) return MOE_ERR_INVALID_ARG;
  if (E > 1024 || topk > 64) return MOE_ERR_BAD_SHAPE;
  if (K % 128 != 0 || N % 128 != 0) return MOE_ERR_BAD_SHAPE;
  if (M * topk > INT32_MAX / 2) return MOE_ERR_BAD_SHAPE;
  return MOE_OK;
}

}  // namespace

size_t fp8_yslots_offset(int64_t M, int E, int topk, int K, int N) { return fp8_layout(M, E, topk, K, N).y; }
}  // namespace moe

extern "C" size_t moe_fused_workspace_bytes_fp8(int64_t num_tokens, int num_experts, int topk, int hidden_size,
                                                int intermediate_size) {
  if (num_tokens < 0 || num_experts <= 0 || topk <= 0 || hidden_size <= 0 || intermediate_size <= 0) return 0;
  return moe::fp8_layout(num_tokens, num_experts, topk, hidden_size, intermediate_size).total;
}

extern "C" int moe_fused_experts_fp8(const void* hidden_states, const void* w1_q, const float* w1_scale,
                                     const void* w2_q, const float* w2_scale, const float* topk_weights,
                                     const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                                     int hidden_size, int intermediate_size, int scale_fmt, void* out,
                                     void* workspace, size_t workspace_bytes, int* status, void* stream) {
  using namespace moe;
  const int64_t M = num_tokens;
  const int E = num_experts, K = hidden_size, N = intermediate_size;
  const int shape = fp8_shape_ok(M, E, topk, K, N);
  if (shape != MOE_OK) return shape;
  if (!scale_fmt_ok(scale_fmt)) return MOE_ERR_INVALID_ARG;
  const bool ue8m0 = scale_fmt == MOE_FP8_SCALE_UE8M0;
  if (M == 0) return MOE_OK;
  if (!hidden_states || !w1_q || !w1_scale || !w2_q || !w2_scale || !topk_weights || !topk_ids || !out || !workspace)
    return MOE_ERR_INVALID_ARG;
  if (!a16(hidden_states) || !a16(w1_q) || !a16(w2_q) || !a16(out) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return MOE_ERR_INVALID_ARG;
  const int dev_ok = moe_check_device();
  if (dev_ok != MOE_OK) return dev_ok;
  const F8Layout2 l = fp8_layout(M, E, topk, K, N);
  if (workspace_bytes < l.total) return MOE_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = launch_quantize_rows(MOE_DTYPE_BF16, hidden_states, M, K, ws + l.xq, K,
                                         reinterpret_cast<float*>(ws + l.xs), K / 128, ue8m0, st);
  if (err == cudaSuccess)
    err = fp8_expert_rows(l, ws, ws + l.xq, K, reinterpret_cast<const float*>(ws + l.xs), K / 128, w1_q, w1_scale,
                          w2_q, w2_scale, topk_weights, topk_ids, M, E, topk, K, N, ue8m0, out, 0, status, st);
  return err == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_fused_experts_fp8_rows(const void* rows, int64_t row_stride, const void* w1_q,
                                          const float* w1_scale, const void* w2_q, const float* w2_scale,
                                          const float* topk_weights, const int32_t* topk_ids, int64_t num_tokens,
                                          int num_experts, int topk, int hidden_size, int intermediate_size,
                                          int scale_fmt, void* out, void* workspace, size_t workspace_bytes,
                                          int max_ctas, int* status, void* stream) {
  using namespace moe;
  const int64_t M = num_tokens;
  const int E = num_experts, K = hidden_size, N = intermediate_size;
  const int shape = fp8_shape_ok(M, E, topk, K, N);
  if (shape != MOE_OK) return shape;
  if (!scale_fmt_ok(scale_fmt)) return MOE_ERR_INVALID_ARG;
  if (row_stride < fp8_row_bytes(K) || row_stride % 16 != 0 || max_ctas < 0) return MOE_ERR_INVALID_ARG;
  if (M == 0) return MOE_OK;
  if (!rows || !w1_q || !w1_scale || !w2_q || !w2_scale || !topk_ids || (out && !topk_weights) || !workspace)
    return MOE_ERR_INVALID_ARG;
  if (!a16(rows) || !a16(w1_q) || !a16(w2_q) || (out && !a16(out)) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return MOE_ERR_INVALID_ARG;
  const int dev_ok = moe_check_device();
  if (dev_ok != MOE_OK) return dev_ok;
  const F8Layout2 l = fp8_layout(M, E, topk, K, N);
  if (workspace_bytes < l.total) return MOE_ERR_WORKSPACE;
  const uint8_t* r = static_cast<const uint8_t*>(rows);
  const cudaError_t err =
      fp8_expert_rows(l, static_cast<uint8_t*>(workspace), r, row_stride, reinterpret_cast<const float*>(r + K),
                      row_stride / 4, w1_q, w1_scale, w2_q, w2_scale, topk_weights, topk_ids, M, E, topk, K, N,
                      scale_fmt == MOE_FP8_SCALE_UE8M0, out, max_ctas, status, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

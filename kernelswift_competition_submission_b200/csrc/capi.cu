// C-ABI entry points that are not a single kernel: device check, status
// strings, and the fused expert path (align -> GEMM1+SiLU*mul -> GEMM2 ->
// top-k combine), all enqueued on the caller's stream with no host sync.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>
#include <mutex>

namespace moe {
namespace {

constexpr int kMaxDevices = 64;

int device_is_sm100() {
  static int cache[kMaxDevices];  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev < 0 || dev >= kMaxDevices) return -1;
  if (cache[dev] == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return -1;
    cache[dev] = (major == 10) ? 1 : 2;
  }
  return cache[dev] == 1 ? 1 : 0;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct FusedLayout {
  size_t meta, sorted, x_sorted, act, y_slots, arrivals, total;
  int64_t cap;
  int64_t n_arrivals;  // [M, n-blocks of the down GEMM] counters of the fused combine
};

FusedLayout fused_layout(int64_t M, int E, int topk, int K, int N) {
  FusedLayout l;
  const int64_t P = M * topk;
  l.cap = moe_align_capacity(P, E, kBlockM);  // each expert's rows padded to whole 128-row m-blocks
  size_t off = 0;
  l.meta = off;     off = align_up(off + sizeof(int32_t) * (size_t)align_meta_ints(E), 256);
  l.sorted = off;   off = align_up(off + sizeof(int32_t) * (size_t)l.cap, 256);
  l.x_sorted = off; off = align_up(off + 2 * (size_t)l.cap * (size_t)K, 256);
  l.act = off;      off = align_up(off + 2 * (size_t)l.cap * (size_t)N, 256);
  l.y_slots = off;  off = align_up(off + 2 * (size_t)P * (size_t)K, 256);
  l.n_arrivals = M * ceil_div(K, gemm2_block_n(K));
  l.arrivals = off; off = align_up(off + sizeof(int32_t) * (size_t)l.n_arrivals, 256);
  l.total = off;
  return l;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

size_t fused_yslots_offset(int64_t M, int E, int topk, int K, int N) { return fused_layout(M, E, topk, K, N).y_slots; }
}  // namespace moe

extern "C" const char* moe_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_BAD_SHAPE: return "unsupported shape";
    case MOE_ERR_UNSUPPORTED: return "unsupported dtype or rule";
    case MOE_ERR_NOT_SM100: return "device is not sm_100 (B200)";
    case MOE_ERR_WORKSPACE: return "workspace too small";
    case MOE_ERR_CUDA: return "CUDA runtime error";
    case MOE_ERR_TIMEOUT: return "device-side wait timed out";
    case MOE_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of the no-allocation entry point";
    default: return "unknown status";
  }
}

extern "C" int moe_abi_version(void) { return 100; }

extern "C" int moe_check_device(void) {
  const int r = moe::device_is_sm100();
  if (r < 0) return MOE_ERR_CUDA;
  return r ? MOE_OK : MOE_ERR_NOT_SM100;
}

extern "C" size_t moe_fused_workspace_bytes(int64_t num_tokens, int num_experts, int topk, int hidden_size,
                                            int intermediate_size) {
  if (num_tokens < 0 || num_experts <= 0 || topk <= 0 || hidden_size <= 0 || intermediate_size <= 0) return 0;
  return moe::fused_layout(num_tokens, num_experts, topk, hidden_size, intermediate_size).total;
}

namespace moe {
namespace {

// Shared argument validation of the expert-path entry points.
int validate_experts(int dtype, int64_t M, int E, int topk, int K, int N) {
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16) return MOE_ERR_UNSUPPORTED;
  if (M < 0 || E <= 0 || topk <= 0 || K <= 0 || N <= 0) return MOE_ERR_INVALID_ARG;
  if (E > 1024 || topk > 64) return MOE_ERR_BAD_SHAPE;
  if (K % 64 != 0 || N % 64 != 0) return MOE_ERR_BAD_SHAPE;
  if (M * topk > INT32_MAX / 2) return MOE_ERR_BAD_SHAPE;
  return MOE_OK;
}

int check_device_ready() {
  const int dev_ok = device_is_sm100();
  if (dev_ok < 0) return MOE_ERR_CUDA;
  return dev_ok ? MOE_OK : MOE_ERR_NOT_SM100;
}

struct Ws {
  int32_t* meta;
  int32_t* sorted;
  void* x_sorted;
  void* act;
  void* y_slots;
  int32_t* arrivals;
  AlignMeta am;
  FusedLayout l;
};

int workspace_views(void* workspace, size_t bytes, int64_t M, int E, int topk, int K, int N, Ws* w) {
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return MOE_ERR_INVALID_ARG;
  w->l = fused_layout(M, E, topk, K, N);
  if (bytes < w->l.total) return MOE_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  w->meta = reinterpret_cast<int32_t*>(ws + w->l.meta);
  w->sorted = reinterpret_cast<int32_t*>(ws + w->l.sorted);
  w->x_sorted = ws + w->l.x_sorted;
  w->act = ws + w->l.act;
  w->y_slots = ws + w->l.y_slots;
  w->arrivals = reinterpret_cast<int32_t*>(ws + w->l.arrivals);
  w->am = align_meta_contiguous(w->meta, E);
  return MOE_OK;
}

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA; }

}  // namespace
}  // namespace moe

extern "C" int moe_expert_align_gather(int dtype, const void* hidden_states, const int32_t* topk_ids,
                                       int64_t num_tokens, int num_experts, int topk, int hidden_size,
                                       int intermediate_size, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!hidden_states || !topk_ids || !aligned16(hidden_states)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  return cuda_status(launch_align(topk_ids, num_tokens * topk, topk, num_experts, kBlockM, w.am, true, w.sorted,
                                  w.l.cap, hidden_states, w.x_sorted, (int64_t)hidden_size * 2,
                                  static_cast<cudaStream_t>(stream)));
}

extern "C" int moe_expert_align(const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                                int hidden_size, int intermediate_size, void* workspace, size_t workspace_bytes,
                                void* stream) {
  using namespace moe;
  int rc = validate_experts(MOE_DTYPE_BF16, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!topk_ids) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  return cuda_status(launch_align(topk_ids, num_tokens * topk, topk, num_experts, kBlockM, w.am, true, w.sorted,
                                  w.l.cap, nullptr, nullptr, 0, static_cast<cudaStream_t>(stream)));
}

extern "C" int moe_expert_gemm1_gather(int dtype, const void* hidden_states, const void* w1, int64_t num_tokens,
                                       int num_experts, int topk, int hidden_size, int intermediate_size,
                                       void* workspace, size_t workspace_bytes, int* status, int max_ctas,
                                       void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!hidden_states || !w1 || !aligned16(hidden_states) || !aligned16(w1)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  return cuda_status(launch_gemm1_gather(dtype, hidden_states, hidden_size, topk, w.sorted, w.l.cap, w1, num_experts,
                                         hidden_size, intermediate_size, w.am.block_start, w.act, status, max_ctas,
                                         static_cast<cudaStream_t>(stream)));
}

extern "C" int moe_expert_gemm1(int dtype, const void* w1, int64_t num_tokens, int num_experts, int topk,
                                int hidden_size, int intermediate_size, void* workspace, size_t workspace_bytes,
                                int* status, int max_ctas, void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!w1 || !aligned16(w1)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  return cuda_status(launch_gemm1_silu(dtype, w.x_sorted, w.l.cap, w1, num_experts, hidden_size, intermediate_size,
                                       w.am.block_start, w.act, status, max_ctas, static_cast<cudaStream_t>(stream)));
}

extern "C" int moe_expert_gemm2(int dtype, const void* w2, int64_t num_tokens, int num_experts, int topk,
                                int hidden_size, int intermediate_size, void* workspace, size_t workspace_bytes,
                                int* status, int max_ctas, void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!w2 || !aligned16(w2)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  return cuda_status(launch_gemm2_scatter(dtype, w.act, w.l.cap, w2, num_experts, hidden_size, intermediate_size,
                                          w.am.block_start, w.sorted, num_tokens * topk, w.y_slots, status, max_ctas,
                                          static_cast<cudaStream_t>(stream)));
}

extern "C" int moe_expert_combine(int dtype, const float* topk_weights, const int32_t* topk_ids, int64_t num_tokens,
                                  int num_experts, int topk, int hidden_size, int intermediate_size, void* out,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!topk_weights || !topk_ids || !out || !aligned16(out)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  return cuda_status(launch_combine(dtype, w.y_slots, topk_weights, topk_ids, num_tokens, topk, num_experts,
                                    hidden_size, out, static_cast<cudaStream_t>(stream)));
}

extern "C" int moe_expert_gemm2_combine(int dtype, const void* w2, const float* topk_weights,
                                        const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                                        int hidden_size, int intermediate_size, void* out, void* workspace,
                                        size_t workspace_bytes, int* status, int max_ctas, void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!w2 || !topk_weights || !topk_ids || !out || !aligned16(w2) || !aligned16(out)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = launch_combine_prep(topk_ids, num_tokens, topk, num_experts, hidden_size, w.arrivals,
                                        w.l.n_arrivals, nullptr, 0, out, st);
  if (err == cudaSuccess)
    err = launch_gemm2_combine(dtype, w.act, w.l.cap, w2, num_experts, hidden_size, intermediate_size,
                               w.am.block_start, w.sorted, w.y_slots, topk_weights, topk_ids, topk, w.arrivals, out,
                               status, max_ctas, st);
  return cuda_status(err);
}

extern "C" int moe_p2p_expert_gemm2_return(int dtype, const void* w2, void* workspace, size_t workspace_bytes,
                                           int num_experts, int hidden_size, int intermediate_size, int topk,
                                           int world, int me, int64_t cap, const int64_t* peer_bases,
                                           const void* own_base, uint32_t seq, int32_t* scratch, int* status,
                                           int max_ctas, void* stream) {
  using namespace moe;
  if (world <= 0 || world > 64 || me < 0 || me >= world || cap <= 0) return MOE_ERR_INVALID_ARG;
  const int64_t M = (int64_t)world * cap;  // every received row, as the align and GEMM1 stages saw them
  int rc = validate_experts(dtype, M, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK) return rc;
  if (!w2 || !aligned16(w2) || !peer_bases || !own_base || !scratch || max_ctas < 0) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, M, num_experts, topk, hidden_size, intermediate_size, &w)) !=
      MOE_OK)
    return rc;
  int64_t offs[9];
  if (moe_p2p_arena_offsets(world, cap, hidden_size, topk, offs) != MOE_OK) return MOE_ERR_INVALID_ARG;
  const char* ob = static_cast<const char*>(own_base);
  const int32_t* own_counts = reinterpret_cast<const int32_t*>(ob + offs[3]);
  const int32_t* recv_id = reinterpret_cast<const int32_t*>(ob + offs[5]);
  const float* recv_w = reinterpret_cast<const float*>(ob + offs[6]);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = launch_combine_prep(recv_id, M, topk, num_experts, hidden_size, w.arrivals, w.l.n_arrivals,
                                        scratch, world, nullptr, st);
  if (err == cudaSuccess)
    err = launch_gemm2_return(dtype, w.act, w.l.cap, w2, num_experts, hidden_size, intermediate_size,
                              w.am.block_start, w.sorted, w.y_slots, recv_w, recv_id, topk, w.arrivals, peer_bases,
                              own_counts, scratch, offs[7], offs[2], cap, me, world, seq, status, max_ctas, st);
  return cuda_status(err);
}

extern "C" int moe_fused_experts(int dtype, const void* hidden_states, const void* w1, const void* w2,
                                 const float* topk_weights, const int32_t* topk_ids, int64_t num_tokens,
                                 int num_experts, int topk, int hidden_size, int intermediate_size, void* out,
                                 void* workspace, size_t workspace_bytes, int* status, void* stream) {
  using namespace moe;
  int rc = validate_experts(dtype, num_tokens, num_experts, topk, hidden_size, intermediate_size);
  if (rc != MOE_OK || num_tokens == 0) return rc;
  if (!hidden_states || !w1 || !w2 || !topk_weights || !topk_ids || !out || !workspace) return MOE_ERR_INVALID_ARG;
  if (!aligned16(hidden_states) || !aligned16(w1) || !aligned16(w2) || !aligned16(out)) return MOE_ERR_INVALID_ARG;
  if ((rc = check_device_ready()) != MOE_OK) return rc;
  Ws w;
  if ((rc = workspace_views(workspace, workspace_bytes, num_tokens, num_experts, topk, hidden_size,
                            intermediate_size, &w)) != MOE_OK)
    return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t P = num_tokens * topk;
  // The measured-fastest stages at every size (the row gather inside GEMM1 and the combine
  // inside GEMM2's epilogue give the same bits but run slower at prefill sizes).
  cudaError_t err = launch_align(topk_ids, P, topk, num_experts, kBlockM, w.am, true, w.sorted, w.l.cap,
                                 hidden_states, w.x_sorted, (int64_t)hidden_size * 2, st);
  if (err == cudaSuccess)
    err = launch_gemm1_silu(dtype, w.x_sorted, w.l.cap, w1, num_experts, hidden_size, intermediate_size,
                            w.am.block_start, w.act, status, 0, st);
  if (err == cudaSuccess)
    err = launch_gemm2_scatter(dtype, w.act, w.l.cap, w2, num_experts, hidden_size, intermediate_size,
                               w.am.block_start, w.sorted, P, w.y_slots, status, 0, st);
  if (err == cudaSuccess)
    err = launch_combine(dtype, w.y_slots, topk_weights, topk_ids, num_tokens, topk, num_experts, hidden_size, out,
                         st);
  return cuda_status(err);
}

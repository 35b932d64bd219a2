// Expert-parallel dispatch / combine helpers (the reference has no multi-GPU
// code; these serve the expert-parallel form of its MoE layer).
//
// A token is sent once to every rank that owns at least one of its top-k
// experts (rank d owns experts [d * epr, (d + 1) * epr), or, with an expert map,
// the experts the map places on d, which lets every rank hold replicas of hot
// experts and keep those pairs at home). Three launches:
//   ep_count_kernel    per-destination row counts (shared-memory histogram of
//                      each token's destination set, then global atomics); the
//                      last CTA scans them into row offsets and also writes the
//                      counts as int64 for the all-to-all split sizes.
//   ep_pack_kernel     warp per token: claims one row per destination, copies
//                      the token's hidden row there (bf16 / fp16, or the packed
//                      e4m3 row: K codes then K / 128 fp32 scales), writes the row's metadata
//                      (k expert ids in the destination's numbering, -1 for
//                      slots it does not own, then the k weights as fp32 bits)
//                      and records where each (token, destination) went.
//   ep_combine_kernel  out[t] = sum over destinations of the returned partial
//                      rows, in fp32, rounded once.
// Row order inside one destination block is unspecified (atomics); every
// returned row is found through the recorded (token, destination) map, so the
// result does not depend on it.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>

namespace moe {
namespace {

constexpr int kEpThreads = 256;
constexpr int kEpMaxWorld = 64;

// Where expert e lives: rank e / epr, local id e % epr, or, with an expert map,
// rank map[e] >> 16 and local id map[e] & 0xffff (ranks holding replicas of hot
// experts route those experts to themselves). Experts outside [0, E) are ignored.
struct ExpertPlace {
  const int32_t* map;
  int epr, E;
  __device__ __forceinline__ bool valid(int e) const { return e >= 0 && e < E; }
  __device__ __forceinline__ int dest(int e) const { return map ? (__ldg(map + e) >> 16) : e / epr; }
  __device__ __forceinline__ int local(int e) const { return map ? (__ldg(map + e) & 0xffff) : e % epr; }
};

__device__ __forceinline__ uint64_t dest_mask(const int32_t* ids_row, int topk, const ExpertPlace& pl) {
  uint64_t m = 0;
  for (int j = 0; j < topk; ++j) {
    const int e = __ldg(ids_row + j);
    if (pl.valid(e)) m |= 1ull << pl.dest(e);
  }
  return m;
}

// meta: [world] counts | [world] cursors | [1] done | [world + 1] offsets (int32), counts64 separate
__global__ void __launch_bounds__(kEpThreads)
ep_count_kernel(const int32_t* __restrict__ ids, int64_t M, int topk, ExpertPlace pl, int world, int32_t* counts,
                int32_t* done, int32_t* offsets, int64_t* counts64) {
  __shared__ int s_cnt[kEpMaxWorld];
  __shared__ int s_last;
  for (int i = threadIdx.x; i < world; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < M; t += (int64_t)gridDim.x * blockDim.x) {
    uint64_t m = dest_mask(ids + t * topk, topk, pl);
    while (m) {
      const int d = __ffsll((long long)m) - 1;
      m &= m - 1;
      atomicAdd(&s_cnt[d], 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < world; i += blockDim.x)
    if (s_cnt[i]) atomicAdd(&counts[i], s_cnt[i]);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(done, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  int run = 0;
  for (int d = 0; d < world; ++d) {
    const int c = __ldcg(&counts[d]);
    offsets[d] = run;
    counts64[d] = c;
    run += c;
  }
  offsets[world] = run;
}

template <typename T>
__global__ void __launch_bounds__(kEpThreads)
ep_pack_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ ids, const float* __restrict__ w, int64_t M,
               int topk, ExpertPlace pl, int world, int64_t row_vecs, const int32_t* __restrict__ offsets, int32_t* cursor,
               uint4* __restrict__ send_x, int32_t* __restrict__ send_meta, int32_t* __restrict__ tok_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= M) return;
  const uint64_t mask = dest_mask(ids + t * topk, topk, pl);
  const int my_e = lane < topk ? __ldg(ids + t * topk + lane) : -1;
  const float my_w = lane < topk ? __ldg(w + t * topk + lane) : 0.f;
  for (int d = 0; d < world; ++d) {
    int row = -1;
    if ((mask >> d) & 1ull) {
      if (lane == 0) row = __ldg(offsets + d) + atomicAdd(&cursor[d], 1);
      row = __shfl_sync(0xffffffffu, row, 0);
      // metadata: ids in d's numbering (-1 if not owned by d), then the weights
      if (lane < topk) {
        const bool own = pl.valid(my_e) && pl.dest(my_e) == d;
        send_meta[(int64_t)row * 2 * topk + lane] = own ? pl.local(my_e) : -1;
        send_meta[(int64_t)row * 2 * topk + topk + lane] = __float_as_int(my_w);
      }
      const uint4* src = x + t * row_vecs;
      uint4* dst = send_x + (int64_t)row * row_vecs;
      for (int64_t v = lane; v < row_vecs; v += 32) dst[v] = __ldg(src + v);
    }
    if (lane == 0) tok_rows[t * world + d] = row;
  }
}

template <typename T>
__global__ void __launch_bounds__(kEpThreads)
ep_combine_kernel(const uint4* __restrict__ back, const int32_t* __restrict__ tok_rows, int64_t M, int world,
                  int vecs_per_row, uint4* __restrict__ out, const int* status) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = gid / vecs_per_row;
  const int v = (int)(gid - t * vecs_per_row);
  if (t >= M) return;
  if (status != nullptr && *reinterpret_cast<const volatile int*>(status) != 0) {
    // the step's transfers failed (a bounded wait gave up): the rows are not this step's
    const uint32_t nan2 = ElemTraits<T>::pack2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
    out[t * vecs_per_row + v] = make_uint4(nan2, nan2, nan2, nan2);
    return;
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int d = 0; d < world; ++d) {
    const int row = __ldg(tok_rows + t * world + d);
    if (row < 0) continue;
    const uint4 q = __ldg(back + (int64_t)row * vecs_per_row + v);
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = ElemTraits<T>::unpack2(u[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  uint4 o;
  o.x = ElemTraits<T>::pack2(acc[0], acc[1]);
  o.y = ElemTraits<T>::pack2(acc[2], acc[3]);
  o.z = ElemTraits<T>::pack2(acc[4], acc[5]);
  o.w = ElemTraits<T>::pack2(acc[6], acc[7]);
  out[t * vecs_per_row + v] = o;
}

inline bool ep_args_ok(int64_t M, int topk, int epr, int world) {
  return M >= 0 && topk > 0 && topk <= 32 && epr > 0 && world > 0 && world <= kEpMaxWorld;
}

}  // namespace

cudaError_t launch_ep_combine(int dtype, const void* back, const int32_t* tok_rows, int64_t M, int K, int world,
                              void* out, const int* status, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  const int vpr = K / 8;
  const unsigned blocks = (unsigned)ceil_div(M * vpr, kEpThreads);
  if (dtype == MOE_DTYPE_BF16)
    ep_combine_kernel<__nv_bfloat16><<<blocks, kEpThreads, 0, st>>>(static_cast<const uint4*>(back), tok_rows, M,
                                                                    world, vpr, static_cast<uint4*>(out), status);
  else
    ep_combine_kernel<__half><<<blocks, kEpThreads, 0, st>>>(static_cast<const uint4*>(back), tok_rows, M, world, vpr,
                                                             static_cast<uint4*>(out), status);
  return cudaGetLastError();
}

}  // namespace moe

extern "C" int64_t moe_ep_send_capacity(int64_t num_tokens, int topk, int world) {
  if (num_tokens < 0 || topk <= 0 || world <= 0) return -1;
  return num_tokens * (int64_t)(topk < world ? topk : world);
}

namespace moe {
namespace {

int ep_plan_impl(const int32_t* topk_ids, int64_t num_tokens, int topk, ExpertPlace pl, int world, int32_t* scratch,
                 int32_t* offsets, int64_t* counts, void* stream) {
  if (!scratch || !offsets || !counts || (num_tokens > 0 && !topk_ids)) return MOE_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // scratch: [world] counts | [world] cursors | [1] done
  if (cudaMemsetAsync(scratch, 0, sizeof(int32_t) * (2 * (size_t)world + 1), st) != cudaSuccess) return MOE_ERR_CUDA;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(num_tokens, kEpThreads), 2 * num_sms()));
  ep_count_kernel<<<blocks, kEpThreads, 0, st>>>(topk_ids, num_tokens, topk, pl, world, scratch, scratch + 2 * world,
                                                 offsets, counts);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int ep_pack_impl(int dtype, const void* hidden_states, const int32_t* topk_ids, const float* topk_weights,
                 int64_t num_tokens, int hidden_size, int topk, ExpertPlace pl, int world, int32_t* scratch,
                 const int32_t* offsets, void* send_x, int32_t* send_meta, int32_t* tok_rows, void* stream) {
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16 && dtype != MOE_DTYPE_E4M3_ROW) return MOE_ERR_UNSUPPORTED;
  if (hidden_size <= 0) return MOE_ERR_INVALID_ARG;
  if (hidden_size % (dtype == MOE_DTYPE_E4M3_ROW ? 128 : 8) != 0) return MOE_ERR_BAD_SHAPE;
  if (num_tokens == 0) return MOE_OK;
  if (!hidden_states || !topk_ids || !topk_weights || !scratch || !offsets || !send_x || !send_meta || !tok_rows)
    return MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(hidden_states) & 15u) || (reinterpret_cast<uintptr_t>(send_x) & 15u))
    return MOE_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)ceil_div(num_tokens * 32, kEpThreads);
  // a row is copied as whole 16-byte vectors: K bf16 / fp16 values, or one packed e4m3 row
  const int64_t row_vecs = (dtype == MOE_DTYPE_E4M3_ROW ? fp8_row_bytes(hidden_size) : (int64_t)hidden_size * 2) / 16;
  if (dtype != MOE_DTYPE_FP16)
    ep_pack_kernel<__nv_bfloat16><<<blocks, kEpThreads, 0, st>>>(
        static_cast<const uint4*>(hidden_states), topk_ids, topk_weights, num_tokens, topk, pl, world, row_vecs,
        offsets, scratch + world, static_cast<uint4*>(send_x), send_meta, tok_rows);
  else
    ep_pack_kernel<__half><<<blocks, kEpThreads, 0, st>>>(
        static_cast<const uint4*>(hidden_states), topk_ids, topk_weights, num_tokens, topk, pl, world, row_vecs,
        offsets, scratch + world, static_cast<uint4*>(send_x), send_meta, tok_rows);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

// expert_map entries: (rank << 16) | local id, rank < world, local id < 65536
bool map_ok(const int32_t* expert_map, int num_experts, int world) {
  return expert_map && num_experts > 0 && world > 0 && world <= kEpMaxWorld;
}

}  // namespace
}  // namespace moe

extern "C" int moe_ep_plan(const int32_t* topk_ids, int64_t num_tokens, int topk, int experts_per_rank, int world,
                           int32_t* scratch, int32_t* offsets, int64_t* counts, void* stream) {
  using namespace moe;
  if (!ep_args_ok(num_tokens, topk, experts_per_rank, world)) return MOE_ERR_INVALID_ARG;
  return ep_plan_impl(topk_ids, num_tokens, topk, ExpertPlace{nullptr, experts_per_rank, experts_per_rank * world},
                      world, scratch, offsets, counts, stream);
}

extern "C" int moe_ep_pack(int dtype, const void* hidden_states, const int32_t* topk_ids, const float* topk_weights,
                           int64_t num_tokens, int hidden_size, int topk, int experts_per_rank, int world,
                           int32_t* scratch, const int32_t* offsets, void* send_x, int32_t* send_meta,
                           int32_t* tok_rows, void* stream) {
  using namespace moe;
  if (!ep_args_ok(num_tokens, topk, experts_per_rank, world)) return MOE_ERR_INVALID_ARG;
  return ep_pack_impl(dtype, hidden_states, topk_ids, topk_weights, num_tokens, hidden_size, topk,
                      ExpertPlace{nullptr, experts_per_rank, experts_per_rank * world}, world, scratch, offsets,
                      send_x, send_meta, tok_rows, stream);
}

extern "C" int moe_ep_plan_mapped(const int32_t* topk_ids, int64_t num_tokens, int topk, int num_experts,
                                  const int32_t* expert_map, int world, int32_t* scratch, int32_t* offsets,
                                  int64_t* counts, void* stream) {
  using namespace moe;
  if (!ep_args_ok(num_tokens, topk, 1, world) || !map_ok(expert_map, num_experts, world)) return MOE_ERR_INVALID_ARG;
  return ep_plan_impl(topk_ids, num_tokens, topk, ExpertPlace{expert_map, 1, num_experts}, world, scratch, offsets,
                      counts, stream);
}

extern "C" int moe_ep_pack_mapped(int dtype, const void* hidden_states, const int32_t* topk_ids,
                                  const float* topk_weights, int64_t num_tokens, int hidden_size, int topk,
                                  int num_experts, const int32_t* expert_map, int world, int32_t* scratch,
                                  const int32_t* offsets, void* send_x, int32_t* send_meta, int32_t* tok_rows,
                                  void* stream) {
  using namespace moe;
  if (!ep_args_ok(num_tokens, topk, 1, world) || !map_ok(expert_map, num_experts, world)) return MOE_ERR_INVALID_ARG;
  return ep_pack_impl(dtype, hidden_states, topk_ids, topk_weights, num_tokens, hidden_size, topk,
                      ExpertPlace{expert_map, 1, num_experts}, world, scratch, offsets, send_x, send_meta, tok_rows,
                      stream);
}

extern "C" int moe_ep_combine(int dtype, const void* returned_rows, const int32_t* tok_rows, int64_t num_tokens,
                              int hidden_size, int world, void* out, void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16) return MOE_ERR_UNSUPPORTED;
  if (num_tokens < 0 || hidden_size <= 0 || world <= 0 || world > kEpMaxWorld) return MOE_ERR_INVALID_ARG;
  if (hidden_size % 8 != 0) return MOE_ERR_BAD_SHAPE;
  if (num_tokens == 0) return MOE_OK;
  if (!returned_rows || !tok_rows || !out) return MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(returned_rows) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u))
    return MOE_ERR_INVALID_ARG;
  return launch_ep_combine(dtype, returned_rows, tok_rows, num_tokens, hidden_size, world, out, nullptr,
                           static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? MOE_OK
             : MOE_ERR_CUDA;
}

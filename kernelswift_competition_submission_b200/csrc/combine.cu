// Top-k combine: out[t] = sum_j topk_weights[t, j] * y[t * topk + j], accumulated in
// fp32 and rounded once to the output type. This is the weighted reduction of
// fused_moe/v0/fused_moe.py:165-167 and the E-reduction kernel of
// fused_moe/v1/fused_moe.py:221-252, reduced over the topk slots instead of all
// experts (the reference's own pending idea, fused_moe/README.md "partial[TOP_K,T,H]").
// Each thread owns 8 consecutive hidden elements (one 16-byte vector) of a token;
// slot rows of a token are contiguous, so every load and store is coalesced, and the
// loads of up to 8 slots are in flight together.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>

namespace moe {
namespace {

template <typename T>
__global__ void __launch_bounds__(256)
combine_kernel(const uint4* __restrict__ y, const float* __restrict__ w, const int32_t* __restrict__ ids, int64_t M,
               int topk, int E, int vecs_per_row, uint4* __restrict__ out) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = gid / vecs_per_row;
  const int v = (int)(gid - t * vecs_per_row);
  if (t >= M) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  // slots in batches of 8: every load of a batch is issued before the first FMA; the FMAs
  // then run in slot order, skipping slots whose expert is outside [0, E)
  for (int j0 = 0; j0 < topk; j0 += 8) {
    uint4 q[8];
    float wj[8];
    bool ok[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      const int e = j < topk ? __ldg(ids + t * topk + j) : -1;
      ok[u] = e >= 0 && e < E;
      wj[u] = ok[u] ? __ldg(w + t * topk + j) : 0.f;
      q[u] = ok[u] ? __ldg(y + (t * topk + j) * vecs_per_row + v) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (!ok[u]) continue;
      const uint32_t h[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = ElemTraits<T>::unpack2(h[i]);
        acc[2 * i] = fmaf(wj[u], f.x, acc[2 * i]);
        acc[2 * i + 1] = fmaf(wj[u], f.y, acc[2 * i + 1]);
      }
    }
  }
  uint4 o;
  o.x = ElemTraits<T>::pack2(acc[0], acc[1]);
  o.y = ElemTraits<T>::pack2(acc[2], acc[3]);
  o.z = ElemTraits<T>::pack2(acc[4], acc[5]);
  o.w = ElemTraits<T>::pack2(acc[6], acc[7]);
  out[t * vecs_per_row + v] = o;
}

// Set-up of the combine fused into the down GEMM (MODE_GEMM2_COMBINE): zeroes the
// [M, NB] arrival counters and `n_zero` further ints (other per-launch counters), and,
// when `out` is given, writes a zero row to it for every token none of whose slots holds
// an expert in [0, E): no GEMM tile reaches such a token, and the reference's expert loop
// leaves its output row at zero (fused_moe/v0/fused_moe.py:154-167).
__global__ void __launch_bounds__(256)
combine_prep_kernel(const int32_t* __restrict__ ids, int64_t M, int topk, int E, int32_t* __restrict__ arrivals,
                    int64_t n_arrivals, int32_t* __restrict__ zero_ints, int n_zero, uint4* __restrict__ out,
                    int vecs_per_row) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t i = gid; i < n_arrivals; i += stride) arrivals[i] = 0;
  for (int64_t i = gid; i < n_zero; i += stride) zero_ints[i] = 0;
  if (out == nullptr) return;  // rows returned elsewhere (expert-parallel return mode)
  for (int64_t t = gid; t < M; t += stride) {
    bool any = false;
    for (int j = 0; j < topk; ++j) {
      const int e = __ldg(ids + t * topk + j);
      any |= (e >= 0 && e < E);
    }
    if (!any)
      for (int v = 0; v < vecs_per_row; ++v) out[t * vecs_per_row + v] = make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace

cudaError_t launch_combine_prep(const int32_t* topk_ids, int64_t M, int topk, int E, int K, int32_t* arrivals,
                                int64_t n_arrivals, int32_t* zero_ints, int n_zero, void* out, cudaStream_t st) {
  const int64_t work = std::max<int64_t>(std::max<int64_t>(n_arrivals, M), n_zero);
  if (work == 0) return cudaSuccess;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(work, 256), 4 * (int64_t)num_sms()));
  combine_prep_kernel<<<blocks, 256, 0, st>>>(topk_ids, M, topk, E, arrivals, n_arrivals, zero_ints, n_zero,
                                              static_cast<uint4*>(out), K / 8);
  return cudaGetLastError();
}

cudaError_t launch_combine(int dtype, const void* y_slots, const float* topk_weights, const int32_t* topk_ids,
                           int64_t M, int topk, int E, int K, void* out, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  const int vpr = K / 8;
  const int64_t threads = M * vpr;
  const unsigned blocks = (unsigned)ceil_div(threads, 256);
  if (dtype == MOE_DTYPE_BF16)
    combine_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const uint4*>(y_slots), topk_weights, topk_ids,
                                                          M, topk, E, vpr, static_cast<uint4*>(out));
  else
    combine_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const uint4*>(y_slots), topk_weights, topk_ids, M,
                                                   topk, E, vpr, static_cast<uint4*>(out));
  return cudaGetLastError();
}

}  // namespace moe

// grouped_topk routing: one warp per token.
//
// Rule (grouped_topk/v0/grouped_topk.py:91-132 of the reference, plus the
// DeepSeek-V3 bias / top-2-sum extension):
//   scores  = softmax(g) | sigmoid(g)
//   choice  = scores (+ bias)
//   gscore  = max(choice in group) | sum of the two largest choice in group
//   keep the topk_group best groups; top-k experts of the kept groups by choice
//   weights = scores of the chosen experts, renormalised, times the scale
// Ordering is the strict total order (value descending, index ascending), the
// rank rule of grouped_topk/v1/grouped_topk.py:94.
//
// Layout: lane l holds experts [l*VPL, l*VPL + VPL) of its token in registers
// (VPL = 8 for E = 256: two 128-bit loads per lane, one coalesced 1 KiB row per
// warp). Group scores go through a per-warp shared-memory row so that any
// group size works; the top-k is k rounds of a warp arg-max over
// (choice, -index) carrying the unbiased score. HBM-bound at large M.
#include "common.cuh"
#include "routing.cuh"

namespace moe {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kMaxExperts = 512;

struct Cand {
  float v;    // ranking value (choice)
  int idx;    // expert index (INT_MAX when empty)
  float s;    // unbiased score (the weight before renormalisation)
};

__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
  return (v1 > v2) || (v1 == v2 && i1 < i2);
}

__device__ __forceinline__ Cand warp_best(Cand c) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Cand o;
    o.v = __shfl_xor_sync(0xffffffffu, c.v, off);
    o.idx = __shfl_xor_sync(0xffffffffu, c.idx, off);
    o.s = __shfl_xor_sync(0xffffffffu, c.s, off);
    if (better(o.v, o.idx, c.v, c.idx)) c = o;
  }
  return c;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <int VPL, bool VEC>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
grouped_topk_kernel(const float* __restrict__ gating, const float* __restrict__ bias, int64_t M, int E,
                    int topk, int renormalize, int n_group, int topk_group, int scoring, int gmode,
                    float scale, float* __restrict__ out_w, int32_t* __restrict__ out_ids) {
  __shared__ float s_choice[kWarpsPerBlock][kMaxExperts];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t tok = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (tok >= M) return;  // whole warp exits together

  const float* row = gating + tok * (int64_t)E;
  const int e0 = lane * VPL;
  float x[VPL];
  if constexpr (VEC) {
#pragma unroll
    for (int i = 0; i < VPL; i += 4) {
      if (e0 + i < E) {
        float4 v = __ldg(reinterpret_cast<const float4*>(row + e0 + i));
        x[i] = v.x; x[i + 1] = v.y; x[i + 2] = v.z; x[i + 3] = v.w;
      } else {
        x[i] = x[i + 1] = x[i + 2] = x[i + 3] = -INFINITY;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) x[i] = (e0 + i < E) ? __ldg(row + e0 + i) : -INFINITY;
  }

  // scores (v0 :98-103)
  float s[VPL];
  if (scoring == MOE_SCORING_SOFTMAX) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPL; ++i) m = fmaxf(m, x[i]);
    m = warp_max(m);
    float z = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      s[i] = (e0 + i < E) ? expf(x[i] - m) : 0.f;
      z += s[i];
    }
    z = warp_sum(z);
#pragma unroll
    for (int i = 0; i < VPL; ++i) s[i] = s[i] / z;
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) s[i] = 1.0f / (1.0f + expf(-x[i]));
  }

  // ranking values
  float c[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const bool valid = e0 + i < E;
    c[i] = valid ? (bias ? s[i] + __ldg(bias + e0 + i) : s[i]) : -INFINITY;
  }

  // group selection (v0 :109-123)
  const int epg = E / n_group;
  if (topk_group < n_group) {
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (e0 + i < E) s_choice[warp][e0 + i] = c[i];
    __syncwarp();
    float gs = -INFINITY;
    if (lane < n_group) {
      const float* gp = &s_choice[warp][lane * epg];
      if (gmode == MOE_GROUP_SCORE_MAX) {
        for (int j = 0; j < epg; ++j) gs = fmaxf(gs, gp[j]);
      } else {
        float b1 = -INFINITY, b2 = -INFINITY;
        for (int j = 0; j < epg; ++j) {
          const float v = gp[j];
          if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) { b2 = v; }
        }
        gs = b1 + b2;
      }
    }
    int rank = 0;
    for (int h = 0; h < n_group; ++h) {
      const float o = __shfl_sync(0xffffffffu, gs, h);
      rank += (o > gs) || (o == gs && h < lane);
    }
    const unsigned keep = __ballot_sync(0xffffffffu, lane < n_group && rank < topk_group);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = e0 + i;
      if (e < E && !((keep >> (e / epg)) & 1u)) c[i] = -INFINITY;
    }
  }

  // top-k rounds (v0 :124)
  unsigned taken = 0;
  float my_w = 0.f;
  int my_id = 0;
  for (int r = 0; r < topk; ++r) {
    Cand b{-INFINITY, INT_MAX, 0.f};
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = e0 + i;
      if (e < E && !((taken >> i) & 1u) && better(c[i], e, b.v, b.idx)) {
        b.v = c[i]; b.idx = e; b.s = s[i];
      }
    }
    b = warp_best(b);
    if (b.idx >= e0 && b.idx < e0 + VPL) taken |= 1u << (b.idx - e0);
    if (lane == r) { my_w = b.s; my_id = b.idx; }
  }

  // renormalise and scale (v0 :126-130)
  if (renormalize) {
    const float tot = warp_sum(lane < topk ? my_w : 0.f);
    my_w = my_w / tot;
  }
  if (scale != 1.0f) my_w *= scale;
  if (lane < topk) {
    out_w[tok * topk + lane] = my_w;
    out_ids[tok * topk + lane] = my_id;
  }
}

template <int VPL, int LPG>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
grouped_topk_lanes_kernel(const float* __restrict__ gating, const float* __restrict__ bias, int64_t M, int topk,
                          int renormalize, int n_group, int topk_group, int scoring, int gmode, float scale,
                          float* __restrict__ out_w, int32_t* __restrict__ out_ids) {
  __shared__ RouteScratch s_scr[kWarpsPerBlock];
  const int64_t tok = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (tok >= M) return;  // whole warp exits together
  route_token_lanes<VPL, LPG, false>(gating + tok * (int64_t)(32 * VPL), bias, tok, topk, renormalize, n_group,
                                     topk_group, scoring, gmode, scale, out_w, out_ids,
                                     &s_scr[threadIdx.x >> 5]);
}

template <int VPL>
cudaError_t launch_vpl(bool vec, const float* g, const float* bias, int64_t M, int E, int topk, int renorm,
                       int n_group, int topk_group, int scoring, int gmode, float scale, float* w,
                       int32_t* ids, cudaStream_t st) {
  const dim3 block(kWarpsPerBlock * 32);
  const dim3 grid((unsigned)ceil_div(M, kWarpsPerBlock));
  if constexpr (VPL % 4 == 0) {
    if (vec) {
      grouped_topk_kernel<VPL, true><<<grid, block, 0, st>>>(g, bias, M, E, topk, renorm, n_group, topk_group,
                                                             scoring, gmode, scale, w, ids);
      return cudaGetLastError();
    }
  }
  grouped_topk_kernel<VPL, false><<<grid, block, 0, st>>>(g, bias, M, E, topk, renorm, n_group, topk_group,
                                                          scoring, gmode, scale, w, ids);
  return cudaGetLastError();
}

}  // namespace
}  // namespace moe

extern "C" int moe_grouped_topk(const float* gating_output, const float* bias, int64_t num_tokens,
                                int num_experts, int topk, int renormalize, int num_expert_group,
                                int topk_group, int scoring_func, int group_score_mode,
                                float routed_scaling_factor, float* topk_weights, int32_t* topk_ids,
                                void* stream) {
  using namespace moe;
  if (num_tokens < 0 || num_experts <= 0 || topk <= 0 || num_expert_group <= 0 || topk_group <= 0)
    return MOE_ERR_INVALID_ARG;
  if (scoring_func != MOE_SCORING_SOFTMAX && scoring_func != MOE_SCORING_SIGMOID) return MOE_ERR_INVALID_ARG;
  if (group_score_mode != MOE_GROUP_SCORE_MAX && group_score_mode != MOE_GROUP_SCORE_TOP2_SUM)
    return MOE_ERR_INVALID_ARG;
  if (num_experts > kMaxExperts || num_expert_group > 32 || topk > 32) return MOE_ERR_BAD_SHAPE;
  if (num_experts % num_expert_group != 0 || topk_group > num_expert_group) return MOE_ERR_BAD_SHAPE;
  const int epg = num_experts / num_expert_group;
  if (topk > topk_group * epg) return MOE_ERR_BAD_SHAPE;
  if (group_score_mode == MOE_GROUP_SCORE_TOP2_SUM && epg < 2) return MOE_ERR_BAD_SHAPE;
  if (num_tokens == 0) return MOE_OK;
  if (!gating_output || !topk_weights || !topk_ids) return MOE_ERR_INVALID_ARG;
  if (num_tokens > (int64_t)INT32_MAX * kWarpsPerBlock) return MOE_ERR_BAD_SHAPE;

  const int vpl_needed = (int)ceil_div(num_experts, 32);
  {
    // register-only variant: every lane full, 16-byte aligned rows, groups of whole lanes
    const bool aligned = ((reinterpret_cast<uintptr_t>(gating_output) & 15u) == 0) &&
                         (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15u) == 0);
    const bool grouped = topk_group < num_expert_group;
    const int lpg = (num_experts / num_expert_group) / 8;  // lanes per group at VPL = 8
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (aligned && num_experts == 256 && topk <= 32 &&
        (!grouped || ((num_experts / num_expert_group) % 8 == 0 && (lpg & (lpg - 1)) == 0))) {
      const dim3 block(kWarpsPerBlock * 32);
      const dim3 grid((unsigned)ceil_div(num_tokens, kWarpsPerBlock));
#define MOE_GTL_ARGS gating_output, bias, num_tokens, topk, renormalize, num_expert_group, topk_group, \
                     scoring_func, group_score_mode, routed_scaling_factor, topk_weights, topk_ids
      switch (grouped ? lpg : 1) {
        case 1: grouped_topk_lanes_kernel<8, 1><<<grid, block, 0, st>>>(MOE_GTL_ARGS); break;
        case 2: grouped_topk_lanes_kernel<8, 2><<<grid, block, 0, st>>>(MOE_GTL_ARGS); break;
        case 4: grouped_topk_lanes_kernel<8, 4><<<grid, block, 0, st>>>(MOE_GTL_ARGS); break;
        case 8: grouped_topk_lanes_kernel<8, 8><<<grid, block, 0, st>>>(MOE_GTL_ARGS); break;
        case 16: grouped_topk_lanes_kernel<8, 16><<<grid, block, 0, st>>>(MOE_GTL_ARGS); break;
        default: grouped_topk_lanes_kernel<8, 32><<<grid, block, 0, st>>>(MOE_GTL_ARGS); break;
      }
#undef MOE_GTL_ARGS
      return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
    }
  }
  const bool vec = (num_experts % 4 == 0) && ((reinterpret_cast<uintptr_t>(gating_output) & 15u) == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err;
#define MOE_GT_ARGS vec, gating_output, bias, num_tokens, num_experts, topk, renormalize, num_expert_group, \
                    topk_group, scoring_func, group_score_mode, routed_scaling_factor, topk_weights, topk_ids, st
  if (vpl_needed <= 1) err = launch_vpl<1>(MOE_GT_ARGS);
  else if (vpl_needed <= 2) err = launch_vpl<2>(MOE_GT_ARGS);
  else if (vpl_needed <= 4) err = launch_vpl<4>(MOE_GT_ARGS);
  else if (vpl_needed <= 8) err = launch_vpl<8>(MOE_GT_ARGS);
  else err = launch_vpl<16>(MOE_GT_ARGS);
#undef MOE_GT_ARGS
  return err == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

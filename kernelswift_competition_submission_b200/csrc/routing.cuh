// Warp-per-token routing rule shared by the grouped_topk kernel and the fused
// router kernel (router GEMM + routing). Rule of grouped_topk/v0/grouped_topk.py:91-132
// of the reference plus the DeepSeek-V3 bias / top-2-sum extension; ordering is the
// strict total order (value descending, index ascending), the rank rule of
// grouped_topk/v1/grouped_topk.py:94.
#pragma once

#include "common.cuh"

namespace moe {

__device__ __forceinline__ bool route_better(float v1, int i1, float v2, int i2) {
  return (v1 > v2) || (v1 == v2 && i1 < i2);
}
__device__ __forceinline__ float route_warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float route_warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Order-preserving map of a float to an unsigned key (a < b as floats <=> key(a) < key(b));
// +0 and -0 map to one key, as they compare equal.
__device__ __forceinline__ unsigned ordered_key(float f) {
  const unsigned u = __float_as_uint(f + 0.0f);  // -0 + 0 = +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit selection key: the value's order-preserving key above the bit-inverted expert
// index, so one unsigned comparison is the strict order (value descending, index
// ascending). 0 is below every real candidate (a real key's high word is never 0).
__device__ __forceinline__ uint64_t route_key(float c, int id) {
  return ((uint64_t)ordered_key(c) << 32) | (uint64_t)(~(uint32_t)id);
}
__device__ __forceinline__ void route_cmpx(uint64_t& a, uint64_t& b) {  // larger key first
  const uint64_t hi = a > b ? a : b;
  const uint64_t lo = a > b ? b : a;
  a = hi;
  b = lo;
}

// Top-k selection for 8 candidates per lane (E = 256): the lane's keys sorted by the
// 19-comparator sorting network for 8 inputs, then per round a warp arg-max of the heads
// (two redux.sync reductions: the high words, then the low words among the lanes that
// hold the largest high word) and a pop of the winner's head. The weight of the chosen
// expert is the lane's score s at that expert, in the unsorted order.
__device__ __forceinline__ void route_select_sorted8(const float (&c)[8], const float (&s)[8], int e0, int lane,
                                                     int64_t tok, int topk, int renormalize, float scale,
                                                     float* __restrict__ out_w, int32_t* __restrict__ out_ids) {
  uint64_t k[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) k[i] = route_key(c[i], e0 + i);
  route_cmpx(k[0], k[2]); route_cmpx(k[1], k[3]); route_cmpx(k[4], k[6]); route_cmpx(k[5], k[7]);
  route_cmpx(k[0], k[4]); route_cmpx(k[1], k[5]); route_cmpx(k[2], k[6]); route_cmpx(k[3], k[7]);
  route_cmpx(k[0], k[1]); route_cmpx(k[2], k[3]); route_cmpx(k[4], k[5]); route_cmpx(k[6], k[7]);
  route_cmpx(k[2], k[4]); route_cmpx(k[3], k[5]);
  route_cmpx(k[1], k[4]); route_cmpx(k[3], k[6]);
  route_cmpx(k[1], k[2]); route_cmpx(k[3], k[4]); route_cmpx(k[5], k[6]);
  float my_w = 0.f;
  int my_id = 0;
  for (int r = 0; r < topk; ++r) {
    const uint32_t hi = (uint32_t)(k[0] >> 32);
    const uint32_t hmax = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t lmax = __reduce_max_sync(0xffffffffu, hi == hmax ? (uint32_t)k[0] : 0u);
    const int bi = (int)(~lmax);
    const int owner = bi >> 3;
    float ws = 0.f;
    if (lane == owner) {
      const int j = bi - e0;  // the winner's score, unsorted order
#pragma unroll
      for (int i = 0; i < 8; ++i) ws = (i == j) ? s[i] : ws;
#pragma unroll
      for (int i = 0; i < 7; ++i) k[i] = k[i + 1];  // pop the head
      k[7] = 0;
    }
    const float bs = __shfl_sync(0xffffffffu, ws, owner);
    if (lane == r) { my_w = bs; my_id = bi; }
  }
  if (renormalize) {
    const float tot = route_warp_sum(lane < topk ? my_w : 0.f);
    my_w = my_w / tot;
  }
  if (scale != 1.0f) my_w *= scale;
  if (lane < topk) {
    out_w[tok * topk + lane] = my_w;
    out_ids[tok * topk + lane] = my_id;
  }
}

// Per-warp shared memory of route_select_threshold8.
struct RouteScratch {
  uint64_t key[32];   // the compacted candidates' selection keys, one per lane
  float c[32];        // compacted candidates: ranking value,
  float s[32];        // score,
  int32_t id[32];     // expert
  float sel_s[32];    // the chosen experts' scores, in rank order
  int32_t sel_id[32]; // the chosen experts, in rank order
};

// Top-k selection by threshold for E = 256 with group masking. Every kept group's two best
// values are >= t (the smallest second-best of the kept groups), and those are
// 2 * topk_group >= topk values, so the k-th best kept value is >= it and nothing below it
// can be chosen. The candidates at or above it (about 8-16 per token for Gaussian logits)
// are compacted one per lane in shared memory; each lane's rank is the number of
// candidates with a larger key (the strict order: value descending, index ascending), and
// ranks 0..topk-1 are the result, in order. Output bits equal route_select_sorted8's: the
// same chosen experts in the same order, the same scores, the same butterfly sum.
// Returns false (nothing written) when more than 32 candidates pass; the caller then runs
// route_select_sorted8.
__device__ __forceinline__ bool route_select_threshold8(const float (&c)[8], const float (&s)[8], int e0, int lane,
                                                        bool kept, float t, int64_t tok, int topk,
                                                        int renormalize, float scale, float* __restrict__ out_w,
                                                        int32_t* __restrict__ out_ids, RouteScratch* scr) {
  // !(c < t): c >= t, or c is NaN (NaN sorts above every number in the key order)
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) m |= (kept && !(c[i] < t)) ? (1u << i) : 0u;
  const int cnt = __popc(m);
  const int n = (int)__reduce_add_sync(0xffffffffu, (unsigned)cnt);
  if (n > 32) return false;
  int pre = cnt;  // inclusive prefix over the lanes
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, pre, off);
    if (lane >= off) pre += v;
  }
  pre -= cnt;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if ((m >> i) & 1u) {
      scr->c[pre] = c[i];
      scr->s[pre] = s[i];
      scr->id[pre] = e0 + i;
      ++pre;
    }
  }
  __syncwarp();
  const uint64_t key = lane < n ? route_key(scr->c[lane], scr->id[lane]) : 0ull;
  const float sv = lane < n ? scr->s[lane] : 0.f;
  scr->key[lane] = key;
  __syncwarp();
  int rank = 0;
  for (int j = 0; j < n; ++j) rank += scr->key[j] > key ? 1 : 0;
  if (lane < n && rank < topk) {
    scr->sel_s[rank] = sv;
    scr->sel_id[rank] = (int32_t)(~(uint32_t)key);
  }
  __syncwarp();
  float my_w = lane < topk ? scr->sel_s[lane] : 0.f;
  const int my_id = lane < topk ? scr->sel_id[lane] : 0;
  __syncwarp();  // the scratch may be reused by this warp's next token
  if (renormalize) {
    const float tot = route_warp_sum(lane < topk ? my_w : 0.f);
    my_w = my_w / tot;
  }
  if (scale != 1.0f) my_w *= scale;
  if (lane < topk) {
    out_w[tok * topk + lane] = my_w;
    out_ids[tok * topk + lane] = my_id;
  }
  return true;
}

// Top-k selection for any VPL: per-lane insertion sort of the candidates (value descending,
// equal values in index order), then per round a warp arg-max of the heads.
template <int VPL>
__device__ __forceinline__ void route_select_insertion(float (&c)[VPL], float (&s)[VPL], int e0, int lane,
                                                       int64_t tok, int topk, int renormalize, float scale,
                                                       float* __restrict__ out_w, int32_t* __restrict__ out_ids) {
  // sort this lane's candidates: value descending; equal values keep index order
  int id[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) id[i] = e0 + i;
#pragma unroll
  for (int i = 1; i < VPL; ++i) {
#pragma unroll
    for (int j = i; j > 0; --j) {
      if (c[j] > c[j - 1]) {
        const float tc = c[j]; c[j] = c[j - 1]; c[j - 1] = tc;
        const float ts = s[j]; s[j] = s[j - 1]; s[j - 1] = ts;
        const int ti = id[j]; id[j] = id[j - 1]; id[j - 1] = ti;
      }
    }
  }

  float my_w = 0.f;
  int my_id = 0;
  for (int r = 0; r < topk; ++r) {
    // warp arg-max of the heads in two reductions: the largest value (as an order-preserving
    // integer key), then the lowest index among the lanes holding it
    const unsigned kmax = __reduce_max_sync(0xffffffffu, ordered_key(c[0]));
    const int bi = (int)__reduce_min_sync(0xffffffffu, ordered_key(c[0]) == kmax ? (unsigned)id[0] : 0xffffffffu);
    const int owner = bi / VPL;
    const float bs = __shfl_sync(0xffffffffu, s[0], owner);
    if (lane == owner) {  // pop the head
#pragma unroll
      for (int i = 0; i + 1 < VPL; ++i) { c[i] = c[i + 1]; s[i] = s[i + 1]; id[i] = id[i + 1]; }
      c[VPL - 1] = -INFINITY;
      id[VPL - 1] = INT_MAX;
    }
    if (lane == r) { my_w = bs; my_id = bi; }
  }

  if (renormalize) {
    const float tot = route_warp_sum(lane < topk ? my_w : 0.f);
    my_w = my_w / tot;
  }
  if (scale != 1.0f) my_w *= scale;
  if (lane < topk) {
    out_w[tok * topk + lane] = my_w;
    out_ids[tok * topk + lane] = my_id;
  }
}

// Register-only variant for the common layouts: E = 32 * VPL (every lane full) and,
// when groups are masked, groups of whole lanes (LPG = E / n_group / VPL lanes per
// group, a power of two): a group's top-2 sum (or max) is a per-lane reduction over
// its VPL values followed by log2(LPG) shuffle steps inside the group's lanes, with no
// shared memory and no serial loop. Each lane then sorts its VPL candidates once
// (value descending, index ascending, the same strict order as above) and each top-k
// round is one warp arg-max over the lanes' current heads (two redux.sync reductions);
// the winner pops its head.
// The scores (weights before renormalisation) travel with the sorted candidates.
// With VPL = 8, group masking, 2 * topk_group >= topk and a per-warp `scr`, the top-k
// is taken by route_select_threshold8 instead (same result, fewer instructions).
// One token's routing by one warp (all 32 lanes); this lane holds the logits x (and the
// bias values bv, when has_bias) of experts [lane * VPL, lane * VPL + VPL).
template <int VPL, int LPG>
__device__ __forceinline__ void route_token_values(const float (&x)[VPL], const float (&bv)[VPL], bool has_bias,
                                                   int64_t tok, int topk, int renormalize, int n_group,
                                                   int topk_group, int scoring, int gmode, float scale,
                                                   float* __restrict__ out_w, int32_t* __restrict__ out_ids,
                                                   RouteScratch* scr) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * VPL;
  float s[VPL];
  if (scoring == MOE_SCORING_SOFTMAX) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPL; ++i) m = fmaxf(m, x[i]);
    m = route_warp_max(m);
    float z = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      s[i] = expf(x[i] - m);
      z += s[i];
    }
    z = route_warp_sum(z);
#pragma unroll
    for (int i = 0; i < VPL; ++i) s[i] = s[i] / z;
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) s[i] = 1.0f / (1.0f + expf(-x[i]));
  }
  float c[VPL];
  if (has_bias) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) c[i] = s[i] + bv[i];
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) c[i] = s[i];
  }

  if (topk_group < n_group) {
    // group score: top-2 sum (or max) of the group's VPL * LPG values
    float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float v = c[i];
      b2 = fmaxf(b2, fminf(b1, v));
      b1 = fmaxf(b1, v);
    }
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, b1, off);
      const float o2 = __shfl_xor_sync(0xffffffffu, b2, off);
      // the two largest of {b1, b2, o1, o2} with b1 >= b2, o1 >= o2
      const float n1 = fmaxf(b1, o1);
      const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
      b1 = n1;
      b2 = n2;
    }
    const float gs = (gmode == MOE_GROUP_SCORE_MAX) ? b1 : b1 + b2;
    const int my_g = lane / LPG;
    // keep the topk_group best groups (score descending, group index ascending): per round
    // the largest remaining score, then the lowest group holding it
    const uint32_t gk = ordered_key(gs);
    bool kept = false;
    for (int r = 0; r < topk_group; ++r) {
      const uint32_t hmax = __reduce_max_sync(0xffffffffu, kept ? 0u : gk);
      const int gmin = (int)__reduce_min_sync(0xffffffffu, (!kept && gk == hmax) ? (unsigned)my_g : 0xffffffffu);
      kept = kept || my_g == gmin;
    }
    if constexpr (VPL == 8) {
      if (scr != nullptr && 2 * topk_group >= topk) {
        const uint32_t tkey = __reduce_min_sync(0xffffffffu, kept ? ordered_key(b2) : 0xffffffffu);
        const float t = __uint_as_float((tkey & 0x80000000u) ? (tkey & 0x7fffffffu) : ~tkey);
        if (route_select_threshold8(c, s, e0, lane, kept, t, tok, topk, renormalize, scale, out_w, out_ids, scr))
          return;
      }
    }
    if (!kept) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) c[i] = -INFINITY;
    }
  }

  if constexpr (VPL == 8) {
    route_select_sorted8(c, s, e0, lane, tok, topk, renormalize, scale, out_w, out_ids);
  } else {
    route_select_insertion<VPL>(c, s, e0, lane, tok, topk, renormalize, scale, out_w, out_ids);
  }
}

// Loads the logits of one token (`row`, E = 32 * VPL floats) and the bias, then applies the
// rule. kCoherent reads the logits through L2 (rows that other CTAs of the same launch
// wrote), otherwise through the read-only path.
template <int VPL>
__device__ __forceinline__ void route_load_row(const float* row, float (&x)[VPL], bool coherent) {
  const int e0 = (threadIdx.x & 31) * VPL;
#pragma unroll
  for (int i = 0; i < VPL; i += 4) {
    const float4 v = coherent ? __ldcg(reinterpret_cast<const float4*>(row + e0 + i))
                              : __ldg(reinterpret_cast<const float4*>(row + e0 + i));
    x[i] = v.x; x[i + 1] = v.y; x[i + 2] = v.z; x[i + 3] = v.w;
  }
}
template <int VPL>
__device__ __forceinline__ void route_load_bias(const float* __restrict__ bias, float (&bv)[VPL]) {
  const int e0 = (threadIdx.x & 31) * VPL;
#pragma unroll
  for (int i = 0; i < VPL; i += 4) {
    const float4 b = bias ? __ldg(reinterpret_cast<const float4*>(bias + e0 + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
    bv[i] = b.x; bv[i + 1] = b.y; bv[i + 2] = b.z; bv[i + 3] = b.w;
  }
}
template <int VPL, int LPG, bool kCoherent>
__device__ __forceinline__ void route_token_lanes(const float* row, const float* __restrict__ bias, int64_t tok,
                                                  int topk, int renormalize, int n_group, int topk_group,
                                                  int scoring, int gmode, float scale, float* __restrict__ out_w,
                                                  int32_t* __restrict__ out_ids, RouteScratch* scr = nullptr) {
  float x[VPL], bv[VPL];
  route_load_row<VPL>(row, x, kCoherent);
  route_load_bias<VPL>(bias, bv);
  route_token_values<VPL, LPG>(x, bv, bias != nullptr, tok, topk, renormalize, n_group, topk_group, scoring, gmode,
                               scale, out_w, out_ids, scr);
}

}  // namespace moe

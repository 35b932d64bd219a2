// Router GEMM fused with grouped_topk: logits = hidden_states . w_gate^T (bf16 or
// fp16 operands, fp32 accumulation on the tensor core) and the routing of every
// token (the rule of routing.cuh) in one launch. The reference starts its path from
// the logits (grouped_topk/v0/grouped_topk.py:93-94 takes gating_output as input);
// this is the step before it, for E = 256 experts.
//
// Grid: one CTA per (128-token m-block, K split). Each CTA runs a K range of the
// 128 x 256 tile through tcgen05 (warp 0: TMA of the hidden rows and of all 256
// gate rows, 64-wide K steps, 4 stages; warp 1: MMA issuer; TMEM accumulator of 256
// fp32 columns), then warps 2-5 move its rows (one per thread) from TMEM to the fp32
// logits: plain stores when the K range is the whole of K, vector reductions
// (red.global.add.v4.f32) into the zeroed logits when the m-block is split. The
// CTAs of an m-block then meet at a per-m-block counter (a cooperative launch when
// the m-block is split, so all are resident; bounded wait) and route its tokens
// together, one warp per token over all 16 warps of each CTA (a token is a long
// dependent chain, so each CTA carries 10 warps that only route), reading the
// logits through L2. Splits give decode-sized batches
// (one m-block) enough CTAs to stream the 3.7 MB of gate weights in parallel.
// All mbarrier waits are bounded (common.cuh).
#include "common.cuh"
#include "moe_internal.h"
#include "routing.cuh"

#include <algorithm>

namespace moe {
namespace {

constexpr int kRThreads = 512;           // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue; all 16 route
constexpr int kRBK = 64;                 // K elements per stage (128 bytes of 16-bit values)
constexpr int kRStages = 4;
constexpr int kRN = 256;                 // experts = MMA N
constexpr int kRATile = kBlockM * kRBK * 2;  // 16 KB
constexpr int kRBTile = kRN * kRBK * 2;      // 32 KB
constexpr int kRStage = kRATile + kRBTile;
constexpr int kRBarOffset = kRStages * kRStage;
constexpr int kRNumBars = 2 * kRStages + 1;
constexpr int kRMiscOffset = kRBarOffset + kRNumBars * 8;
constexpr int kRSmem = 1024 + kRMiscOffset + 16;

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

template <typename T, int LPG>
__global__ void __launch_bounds__(kRThreads, 1)
router_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int64_t M,
              int K, int splits, float* __restrict__ logits, int* __restrict__ mb_done,
              const float* __restrict__ bias, int topk, int renormalize, int n_group, int topk_group, int scoring,
              int gmode, float scale, float* __restrict__ out_w, int32_t* __restrict__ out_ids, int* status) {
  constexpr uint32_t kIdesc = idesc_f16(kBlockM, kRN, ElemTraits<T>::kFmt);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRBarOffset);
  uint64_t* empty = full + kRStages;
  uint64_t* acc_full = full + 2 * kRStages;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + kRMiscOffset);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kRMiscOffset + 4);
  int* s_last = reinterpret_cast<int*>(smem + kRMiscOffset + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mb = blockIdx.x / splits;
  const int sp = blockIdx.x - mb * splits;
  const int kt = K / kRBK;
  const int per = (kt + splits - 1) / splits;
  const int k0 = sp * per;
  const int k1 = min(kt, k0 + per);
  const bool has_work = k0 < k1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(acc_full, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&map_a); tma_prefetch_desc(&map_b); }
  if (warp == 2) { tmem_alloc(s_tmem, kRN); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (warp == 0) {
    if (lane == 0 && has_work) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int kb = k0; kb < k1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
        uint8_t* a_dst = smem + stage * kRStage;
        mbar_arrive_expect_tx(&full[stage], kRStage);
        tma_load_2d(&map_a, &full[stage], a_dst, kb * kRBK, mb * kBlockM);
        tma_load_2d(&map_b, &full[stage], a_dst + kRATile, kb * kRBK, 0);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kRStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) {
        for (int s = 0; s < kRStages; ++s)
          if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && has_work) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = k0; kb < k1; ++kb) {
        if (!mbar_wait(&full[stage], phase, status, s_abort)) { ok = false; break; }
        tc_fence_after();
        const uint8_t* a_src = smem + stage * kRStage;
        const uint64_t a_desc = smem_desc_sw128(a_src);
        const uint64_t b_desc = smem_desc_sw128(a_src + kRATile);
#pragma unroll
        for (int k = 0; k < kRBK / 16; ++k)
          umma_f16(tmem_base, a_desc + 2 * k, b_desc + 2 * k, kIdesc, (kb > k0 || k > 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == kRStages) { stage = 0; phase ^= 1; }
      }
      umma_commit(acc_full);  // also when aborted: the epilogue's wait then ends
      mbar_wait(acc_full, 0, nullptr, nullptr);  // no TMEM release before the MMAs completed
      (void)ok;
    }
  } else if (warp < 6 && has_work) {
    // ------------------------------------------------ TMEM -> logits (warps 2-5)
    const int quad = warp & 3;
    const int64_t grow = (int64_t)mb * kBlockM + quad * 32 + lane;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, status, s_abort));
    if (ok) {
      tc_fence_after();
      float* dst = logits + grow * kRN;
#pragma unroll 1
      for (int c = 0; c < kRN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + c * 32, v);
        tmem_wait_ld();
        if (grow < M) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float a = __uint_as_float(v[i]), b = __uint_as_float(v[i + 1]);
            const float cc = __uint_as_float(v[i + 2]), d = __uint_as_float(v[i + 3]);
            if (splits == 1)
              *reinterpret_cast<float4*>(dst + c * 32 + i) = make_float4(a, b, cc, d);
            else
              red_add_v4(dst + c * 32 + i, a, b, cc, d);
          }
        }
      }
    }
  }

  // ------------------------------------------------ routing, shared by the m-block's CTAs
  // Every CTA of the m-block publishes its part (counter), waits for the others (the
  // launch is cooperative when an m-block is split, so they are all resident; the wait
  // is bounded all the same) and routes every splits-th token of the m-block.
  tc_fence_before();
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicAdd(mb_done + mb, 1);
    int ready = 1;
    if (splits > 1) {
      const uint64_t t0 = globaltimer_ns();
      while (true) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(mb_done + mb) : "memory");
        if (v >= splits) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          record_status(status, MOE_ERR_TIMEOUT);
          ready = 0;
          break;
        }
        __nanosleep(256);
      }
    }
    *s_last = ready && *s_abort == 0;
  }
  __syncthreads();
  if (*s_last) {
    __threadfence();
    const int64_t t_end = M < (int64_t)(mb + 1) * kBlockM ? M : (int64_t)(mb + 1) * kBlockM;
    // the stage buffers are idle now (every load was consumed by a finished MMA): one
    // routing scratch per warp at their start
    RouteScratch* scr = reinterpret_cast<RouteScratch*>(smem) + warp;
    for (int64_t tok = (int64_t)mb * kBlockM + sp + (int64_t)warp * splits; tok < t_end;
         tok += (int64_t)(kRThreads / 32) * splits)
      route_token_lanes<8, LPG, true>(logits + tok * kRN, bias, tok, topk, renormalize, n_group, topk_group,
                                      scoring, gmode, scale, out_w, out_ids, scr);
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kRN);
  }
}

template <typename T, int LPG>
cudaError_t launch_router(const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int K, int splits, int grid,
                          float* logits, int* done, const float* bias, int topk, int renorm, int n_group,
                          int topk_group, int scoring, int gmode, float scale, float* w, int32_t* ids, int* status,
                          cudaStream_t st) {
  auto kern = router_kernel<T, LPG>;
  cudaError_t err = ensure_smem_limit(reinterpret_cast<const void*>(kern), kRSmem);
  if (err != cudaSuccess) return err;
  if (splits == 1) {
    kern<<<grid, kRThreads, kRSmem, st>>>(ma, mb, M, K, splits, logits, done, bias, topk, renorm, n_group,
                                          topk_group, scoring, gmode, scale, w, ids, status);
    return cudaGetLastError();
  }
  // split m-blocks wait for one another: a cooperative launch guarantees co-residency
  int64_t M_ = M;
  int K_ = K, splits_ = splits, topk_ = topk, renorm_ = renorm, ng_ = n_group, tg_ = topk_group, sc_ = scoring,
      gm_ = gmode;
  float scale_ = scale;
  void* args[] = {const_cast<CUtensorMap*>(&ma), const_cast<CUtensorMap*>(&mb), &M_, &K_, &splits_, &logits, &done,
                  const_cast<float**>(&bias), &topk_, &renorm_, &ng_, &tg_, &sc_, &gm_, &scale_, &w, &ids, &status};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kRThreads), args, kRSmem,
                                     st);
}

}  // namespace
}  // namespace moe

extern "C" int64_t moe_router_scratch_ints(int64_t num_tokens) {
  return num_tokens < 0 ? -1 : (num_tokens + moe::kBlockM - 1) / moe::kBlockM;
}

extern "C" int moe_router_grouped_topk(int dtype, const void* hidden_states, const void* w_gate, const float* bias,
                                       int64_t num_tokens, int num_experts, int hidden_size, int topk,
                                       int renormalize, int num_expert_group, int topk_group, int scoring_func,
                                       int group_score_mode, float routed_scaling_factor, float* logits_out,
                                       float* topk_weights, int32_t* topk_ids, int32_t* scratch, int* status,
                                       void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16) return MOE_ERR_UNSUPPORTED;
  if (num_tokens < 0 || hidden_size <= 0 || topk <= 0 || num_expert_group <= 0 || topk_group <= 0)
    return MOE_ERR_INVALID_ARG;
  if (scoring_func != MOE_SCORING_SOFTMAX && scoring_func != MOE_SCORING_SIGMOID) return MOE_ERR_INVALID_ARG;
  if (group_score_mode != MOE_GROUP_SCORE_MAX && group_score_mode != MOE_GROUP_SCORE_TOP2_SUM)
    return MOE_ERR_INVALID_ARG;
  // the tile is all 256 experts; groups must be whole lanes of the routing warp (8 experts per lane)
  if (num_experts != 256 || hidden_size % 64 != 0 || topk > 32) return MOE_ERR_BAD_SHAPE;
  if (num_experts % num_expert_group != 0 || topk_group > num_expert_group) return MOE_ERR_BAD_SHAPE;
  const int epg = num_experts / num_expert_group;
  const bool grouped = topk_group < num_expert_group;
  const int lpg = grouped ? epg / 8 : 1;
  if (grouped && (epg % 8 != 0 || (lpg & (lpg - 1)) != 0)) return MOE_ERR_BAD_SHAPE;
  if (topk > topk_group * epg) return MOE_ERR_BAD_SHAPE;
  if (group_score_mode == MOE_GROUP_SCORE_TOP2_SUM && epg < 2) return MOE_ERR_BAD_SHAPE;
  if (num_tokens == 0) return MOE_OK;
  if (!hidden_states || !w_gate || !logits_out || !topk_weights || !topk_ids || !scratch) return MOE_ERR_INVALID_ARG;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(hidden_states) || !a16(w_gate) || !a16(logits_out) || (bias && !a16(bias))) return MOE_ERR_INVALID_ARG;
  const int dev_ok = moe_check_device();
  if (dev_ok != MOE_OK) return dev_ok;

  const int64_t mblocks = (num_tokens + kBlockM - 1) / kBlockM;
  if (mblocks > INT32_MAX / 64) return MOE_ERR_BAD_SHAPE;
  const int kt = hidden_size / kRBK;
  // enough CTAs to cover the SMs, at least 4 K steps per split
  int splits = (int)std::max<int64_t>(1, num_sms() / mblocks);
  splits = std::max(1, std::min(splits, kt / 4));
  const int per = (kt + splits - 1) / splits;
  splits = (kt + per - 1) / per;  // no empty split
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, sizeof(int32_t) * mblocks, st) != cudaSuccess) return MOE_ERR_CUDA;
  if (splits > 1 &&
      cudaMemsetAsync(logits_out, 0, sizeof(float) * (size_t)num_tokens * kRN, st) != cudaSuccess)
    return MOE_ERR_CUDA;

  CUtensorMap ma, mbm;
  const uint64_t a_dims[2] = {(uint64_t)hidden_size, (uint64_t)num_tokens};
  const uint64_t a_str[1] = {(uint64_t)hidden_size * 2};
  const uint64_t b_dims[2] = {(uint64_t)hidden_size, (uint64_t)kRN};
  if (!make_kmajor_map(&ma, dtype, hidden_states, 2, a_dims, a_str, kBlockM)) return MOE_ERR_CUDA;
  if (!make_kmajor_map(&mbm, dtype, w_gate, 2, b_dims, a_str, kRN)) return MOE_ERR_CUDA;
  const int grid = (int)(mblocks * splits);
  cudaError_t err = cudaErrorInvalidValue;
#define MOE_R_ARGS ma, mbm, num_tokens, hidden_size, splits, grid, logits_out, scratch, bias, topk, renormalize, \
                   num_expert_group, topk_group, scoring_func, group_score_mode, routed_scaling_factor, topk_weights, \
                   topk_ids, status, st
#define MOE_R_LPG(T)                                                   \
  switch (lpg) {                                                       \
    case 1: err = launch_router<T, 1>(MOE_R_ARGS); break;              \
    case 2: err = launch_router<T, 2>(MOE_R_ARGS); break;              \
    case 4: err = launch_router<T, 4>(MOE_R_ARGS); break;              \
    case 8: err = launch_router<T, 8>(MOE_R_ARGS); break;              \
    case 16: err = launch_router<T, 16>(MOE_R_ARGS); break;            \
    default: err = launch_router<T, 32>(MOE_R_ARGS); break;            \
  }
  if (dtype == MOE_DTYPE_BF16) { MOE_R_LPG(__nv_bfloat16) } else { MOE_R_LPG(__half) }
#undef MOE_R_LPG
#undef MOE_R_ARGS
  return err == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

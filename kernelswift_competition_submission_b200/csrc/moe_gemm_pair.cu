// Grouped expert GEMMs on pairs of SMs: tcgen05.mma.cta_group::2, TMEM
// accumulators, TMA-fed operands, swap-AB.
//
// The two expert GEMMs of fused_moe/v0/fused_moe.py:160-163 are computed
// transposed, with the expert WEIGHTS as the MMA's M operand and the TOKENS as
// its N operand:
//   GEMM1_SILU  act[t, f] = silu(w1[e, f] . x_t) * (w1[e, N + f] . x_t)     (:160-162)
//   GEMM2       y[pair(t), f] = w2[e, f] . act_t                             (:163)
// Rows t are the (token, slot) pairs grouped by expert by the align stage,
// with no padding: expert e owns rows [off[e], off[e+1]).
//
// Why swap-AB on a CTA pair:
//   * M = 256 weight rows per tile, split 128/128 over the two CTAs of a
//     cluster; N = T tokens (T <= 256, a multiple of 32 chosen per tile), split
//     T/2 + T/2. Each CTA stages 32 KB per 64-wide K step for a 128 x T x 64 MMA
//     slice instead of 48 KB for the 1-CTA 128 x 256 tile.
//   * The expert's token count only needs rounding to 32, not to the 128 or
//     256 rows a token-major tile wastes; decode-sized batches (1..8 tokens per
//     expert) run as T = 32 tiles that stream the weights once.
//   * GEMM1's SiLU*mul pairs gate feature f with up feature f: each CTA's A half
//     stacks 64 gate rows over the 64 matching up rows, so both land in the
//     same CTA's TMEM (lanes 0-63 gate, 64-127 up) and meet in shared memory.
//
// Roles (256 threads per CTA, one CTA pair per cluster, persistent):
//   warp 0      TMA producer, both CTAs: loads its A half (weights) and B half
//               (tokens) of each stage; bytes are counted on the LEADER CTA's
//               `full` barrier (.cta_group::2).
//   warp 1      MMA issuer, leader CTA only: 4 x tcgen05.mma.cta_group::2 per
//               stage; commits release the stage in both CTAs (multicast) and,
//               per tile, mark the accumulator full in both CTAs.
//   warp 2      TMEM allocator (cta_group::2, 2 accumulators x 256 columns).
//   warp 3      computes the per-expert tile prefix in the prologue.
//   warps 4-7   epilogue, both CTAs: TMEM -> registers (one feature per
//               thread, 32 tokens per load) -> shared memory transpose ->
//               coalesced 16-byte global stores of whole token rows; arrive
//               on the leader's `tmem_empty` so the next tile's MMAs can reuse
//               the accumulator while this one is stored.
// No TMA multicast: every CTA loads its own operands.
// All mbarrier waits are bounded (common.cuh). On a timeout every role stops,
// the leader's producer waits (bounded) for the copies in flight, the MMA thread
// waits for its MMAs, the pair meets at a cluster barrier and frees TMEM.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>

namespace moe {
namespace {

enum { PAIR_GEMM1_SILU = 0, PAIR_GEMM2 = 1 };

constexpr int kPThreads = 256;
constexpr int kTokTile = 256;        // max tokens (N) per pair tile
constexpr int kPBK = 64;             // K elements per stage (128 bytes)
constexpr int kPStages = 6;
constexpr int kAHalf = 128 * kPBK * 2;   // 16 KB: this CTA's 128 weight rows
constexpr int kBHalf = 128 * kPBK * 2;   // 16 KB: up to 128 token rows
constexpr int kPStage = kAHalf + kBHalf;
constexpr int kEpiBytes = 64 * 33 * 4 + 32 * 128 * 2;  // GEMM1 up buffer + out tile (>= GEMM2's 8 KB tile)
constexpr int kEpiOffset = kPStages * kPStage;
constexpr int kBarOffset = kEpiOffset + kEpiBytes;
constexpr int kNumBars = 2 * kPStages + 5;
constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
constexpr int kTablesOffset = kMiscOffset + 16;
inline int pair_smem_bytes(int E) { return 1024 + kTablesOffset + 12 * (E + 1); }

struct PairTile {
  int e, fb, t0, valid, T;
};

// Tile order: every full 256-token tile of every expert first (expert-major,
// then feature block, token block fastest), then the partial tail tiles. Tiles
// running at the same time are then equally long, so the CTA pairs stay in
// step and the operands they share (an expert's weight block across its token
// blocks, a token block across the feature blocks) are reused from L2 instead
// of being re-read from HBM by pairs that drifted apart.
__device__ __forceinline__ int find_expert(const int* s_pre, int E, int tile) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_pre[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ PairTile decode_pair_tile(const int* s_off, const int* s_full, const int* s_tail, int E,
                                                     int FB, int tile) {
  PairTile p;
  const int total_full = s_full[E];
  if (tile < total_full) {
    p.e = find_expert(s_full, E, tile);
    const int nfull = (s_off[p.e + 1] - s_off[p.e]) / kTokTile;
    const int local = tile - s_full[p.e];
    p.fb = local / nfull;
    const int tb = local - p.fb * nfull;
    p.t0 = s_off[p.e] + tb * kTokTile;
    p.valid = kTokTile;
  } else {
    const int t2 = tile - total_full;
    p.e = find_expert(s_tail, E, t2);
    const int cnt = s_off[p.e + 1] - s_off[p.e];
    p.fb = t2 - s_tail[p.e];
    p.t0 = s_off[p.e] + (cnt / kTokTile) * kTokTile;
    p.valid = cnt % kTokTile;
  }
  p.T = (p.valid + 31) & ~31;
  return p;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kPThreads, 1)
moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_b16, const int32_t* __restrict__ expert_off, int E,
                     int k_red, int n_feat, int FB, T* __restrict__ out, const int32_t* __restrict__ sorted_pairs,
                     int* status) {
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOffset);
  uint64_t* empty = full + kPStages;
  uint64_t* tmem_full = full + 2 * kPStages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_done = tmem_full + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + kMiscOffset);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kMiscOffset + 4);
  int* s_off = reinterpret_cast<int*>(smem + kTablesOffset);
  int* s_full = s_off + (E + 1);   // prefix over experts of full-tile counts
  int* s_tail = s_full + (E + 1);  // prefix over experts of tail-tile counts
  float* up_buf = reinterpret_cast<float*>(smem + kEpiOffset);                       // [64][33] fp32
  T* out_tile = reinterpret_cast<T*>(smem + kEpiOffset + 64 * 33 * 4);                // [32][64] or [32][128]
  T* out_tile2 = reinterpret_cast<T*>(smem + kEpiOffset);                              // GEMM2: [32][128]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();  // 0 = leader of the pair
  const bool leader = (cta == 0);

  // ---------------- prologue
  for (int i = threadIdx.x; i <= E; i += kPThreads) s_off[i] = __ldg(expert_off + i);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tmem_full[a], 1); mbar_init(&tmem_empty[a], 8); }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_b16);
  }
  if (warp == 2) { tmem_alloc_pair(s_tmem, kTmemCols); tmem_relinquish_pair(); }
  __syncthreads();  // s_off visible to warp 3
  if (warp == 3) {
    // s_full[e] = sum over e' < e of floor(count / 256) * FB, s_tail[e] = sum of (count % 256 != 0) * FB
    const int per = (E + 31) / 32;
    const int b = lane * per;
    int lf = 0, lt = 0;
    for (int i = 0; i < per; ++i) {
      if (b + i < E) {
        const int cnt = s_off[b + i + 1] - s_off[b + i];
        lf += (cnt / kTokTile) * FB;
        lt += (cnt % kTokTile != 0) * FB;
      }
    }
    int inf = lf, int_ = lt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int vf = __shfl_up_sync(0xffffffffu, inf, o);
      const int vt = __shfl_up_sync(0xffffffffu, int_, o);
      if (lane >= o) { inf += vf; int_ += vt; }
    }
    int rf = inf - lf, rt = int_ - lt;
    for (int i = 0; i < per; ++i) {
      if (b + i < E) {
        const int cnt = s_off[b + i + 1] - s_off[b + i];
        s_full[b + i] = rf;
        s_tail[b + i] = rt;
        rf += (cnt / kTokTile) * FB;
        rt += (cnt % kTokTile != 0) * FB;
      }
    }
    if (lane == 31) { s_full[E] = inf; s_tail[E] = int_; }
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits, TMEM address and tables visible across the pair
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_tiles = s_full[E] + s_tail[E];
  const int num_kb = (k_red + kPBK - 1) / kPBK;
  const int pair_id = (int)cluster_id_x();
  const int num_pairs = (int)num_clusters_x();
  bool producer_aborted = false;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = pair_id; tile < total_tiles && ok; tile += num_pairs) {
        const PairTile pt = decode_pair_tile(s_off, s_full, s_tail, E, FB, tile);
        const int half_t = pt.T >> 1;
        const uint32_t b_bytes = (pt.T == kTokTile) ? (uint32_t)kBHalf : (uint32_t)(half_t * kPBK * 2);
        const int row0 = pt.t0 + (int)cta * half_t;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
          uint8_t* a_dst = smem + stage * kPStage;
          uint8_t* b_dst = a_dst + kAHalf;
          const int kc = kb * kPBK;
          const uint32_t full_leader = mapa_shared(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2u * ((uint32_t)kAHalf + b_bytes));
          if constexpr (MODE == PAIR_GEMM1_SILU) {
            const int f0 = pt.fb * 128 + 64 * (int)cta;
            tma_load_3d_pair(&map_a, full_leader, a_dst, kc, f0, 2 * pt.e);
            tma_load_3d_pair(&map_a, full_leader, a_dst + 64 * kPBK * 2, kc, f0, 2 * pt.e + 1);
          } else {
            tma_load_3d_pair(&map_a, full_leader, a_dst, kc, pt.fb * 256 + 128 * (int)cta, pt.e);
          }
          if (pt.T == kTokTile) {
            tma_load_2d_pair(&map_b, full_leader, b_dst, kc, row0);
          } else {
            for (int i = 0; i < half_t; i += 16) tma_load_2d_pair(&map_b16, full_leader, b_dst + i * kPBK * 2, kc, row0 + i);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kPStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        producer_aborted = true;
        // drain: the leader's `full` barriers count both CTAs' bytes, so the leader
        // waits (bounded, ignoring the abort flag) for the last phase it armed.
        if (leader) {
          for (int s = 0; s < kPStages; ++s)
            if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------ MMA issuer (leader CTA)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair_id; tile < total_tiles && ok; tile += num_pairs) {
        const PairTile pt = decode_pair_tile(s_off, s_full, s_tail, E, FB, tile);
        const uint32_t idesc = idesc_f16(256, pt.T, ElemTraits<T>::kFmt);
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, status, s_abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kTokTile);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* a_src = smem + stage * kPStage;
          const uint64_t a_desc = smem_desc_sw128(a_src);
          const uint64_t b_desc = smem_desc_sw128(a_src + kAHalf);
#pragma unroll
          for (int k = 0; k < kPBK / 16; ++k)
            umma_f16_pair(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair_multicast(&empty[stage], 0x3);
          if (++stage == kPStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair_multicast(&tmem_full[acc], 0x3);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit_pair(mma_done);
      mbar_wait(mma_done, 0, nullptr, nullptr);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 4;           // TMEM lanes 32*ew .. +31
    const int et = threadIdx.x - 128;  // 0..127
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair_id; tile < total_tiles; tile += num_pairs) {
      const PairTile pt = decode_pair_tile(s_off, s_full, s_tail, E, FB, tile);
      const bool got = __all_sync(0xffffffffu, mbar_wait(&tmem_full[acc], acc_phase, status, s_abort));
      if (!named_bar_and(1, 128, got)) break;  // all four epilogue warps leave together
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * kTokTile);
      const int nchunks = pt.T >> 5;
      for (int c = 0; c < nchunks; ++c) {
        uint32_t v[32];
        tmem_ld32(t_row + c * 32, v);
        tmem_wait_ld();
        if (c == nchunks - 1) {
          // accumulator fully read: hand it back to the leader's MMA thread
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(&tmem_empty[acc], 0));
        }
        if constexpr (MODE == PAIR_GEMM1_SILU) {
          if (ew >= 2) {
            float* u = up_buf + (32 * (ew - 2) + lane) * 33;
#pragma unroll
            for (int j = 0; j < 32; ++j) u[j] = __uint_as_float(v[j]);
          }
          named_bar_sync(1, 128);
          if (ew < 2) {
            const int fi = 32 * ew + lane;
            const float* u = up_buf + fi * 33;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float g = __uint_as_float(v[j]);
              const float a = g / (1.0f + __expf(-g)) * u[j];
              out_tile[j * 64 + fi] = ElemTraits<T>::from_float(a);
            }
          }
          named_bar_sync(1, 128);
          // 32 token rows x 64 features (128 B) -> act rows
          const int fbase = pt.fb * 128 + 64 * (int)cta;
          if (fbase < n_feat) {
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int ch = et + 128 * q;
              const int r = ch >> 3, col = ch & 7;
              if (c * 32 + r < pt.valid) {
                const uint4 val = *reinterpret_cast<const uint4*>(out_tile + r * 64 + col * 8);
                *reinterpret_cast<uint4*>(out + (int64_t)(pt.t0 + c * 32 + r) * n_feat + fbase + col * 8) = val;
              }
            }
          }
          named_bar_sync(1, 128);
        } else {
          const int fi = 32 * ew + lane;  // 0..127
#pragma unroll
          for (int j = 0; j < 32; ++j) out_tile2[j * 128 + fi] = ElemTraits<T>::from_float(__uint_as_float(v[j]));
          named_bar_sync(1, 128);
          // 32 token rows x 128 features (256 B) -> slot rows of their pairs
          const int fbase = pt.fb * 256 + 128 * (int)cta;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int ch = et + 128 * q;
            const int r = ch >> 4, col = ch & 15;
            const int f = fbase + col * 8;
            if (c * 32 + r < pt.valid && f < n_feat) {
              const int pair = __ldg(sorted_pairs + pt.t0 + c * 32 + r);
              const uint4 val = *reinterpret_cast<const uint4*>(out_tile2 + r * 128 + col * 8);
              if (pair >= 0) *reinterpret_cast<uint4*>(out + (int64_t)pair * n_feat + f) = val;
            }
          }
          named_bar_sync(1, 128);
        }
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  if (producer_aborted && !leader) {
    // the peer cannot observe its own copies completing (they count on the leader's
    // barrier); give copies in flight a bounded grace period before the pair exits
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its barriers or TMEM
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
template <typename T, int MODE>
cudaError_t launch_pair_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb16, const int32_t* off,
                          int E, int k_red, int n_feat, int FB, int64_t num_pairs_rows, void* out,
                          const int32_t* sorted_pairs, int* status, cudaStream_t st) {
  auto kern = moe_gemm_pair_kernel<T, MODE>;
  const int smem = pair_smem_bytes(E);
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Persistent grid of exactly the CTA pairs that can be resident at once: a pair
  // needs two SMs of one GPC, so not every SM can host one; a pair launched beyond
  // that would start late and run out of step with the others.
  cfg.gridDim = dim3(num_sms(), 1, 1);
  int resident = 0;
  if (cudaOccupancyMaxActiveClusters(&resident, kern, &cfg) != cudaSuccess || resident <= 0) resident = num_sms() / 2;
  const int64_t tiles_cap = (ceil_div(num_pairs_rows, kTokTile) + E) * (int64_t)FB;
  const int clusters = (int)std::max<int64_t>(1, std::min<int64_t>(resident, tiles_cap));
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, mb16, off, E, k_red, n_feat, FB, static_cast<T*>(out), sorted_pairs,
                            status);
}

}  // namespace

bool make_kmajor_map(CUtensorMap* m, int dtype, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, uint32_t box_rows);

cudaError_t launch_pair_gemm1_silu(int dtype, const void* x_sorted, int64_t P, const void* w1, int E, int K, int N,
                                   const int32_t* expert_off, void* act, int* status, cudaStream_t st) {
  CUtensorMap ma, mb, mb16;
  const uint64_t a_dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)2 * E};
  const uint64_t a_str[2] = {(uint64_t)K * 2, (uint64_t)N * K * 2};
  const uint64_t b_dims[2] = {(uint64_t)K, (uint64_t)P};
  const uint64_t b_str[1] = {(uint64_t)K * 2};
  if (!make_kmajor_map(&ma, dtype, w1, 3, a_dims, a_str, 64)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mb, dtype, x_sorted, 2, b_dims, b_str, 128)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mb16, dtype, x_sorted, 2, b_dims, b_str, 16)) return cudaErrorInvalidValue;
  const int FB = (int)ceil_div(N, 128);
  if (dtype == MOE_DTYPE_BF16)
    return launch_pair_t<__nv_bfloat16, PAIR_GEMM1_SILU>(ma, mb, mb16, expert_off, E, K, N, FB, P, act, nullptr,
                                                         status, st);
  return launch_pair_t<__half, PAIR_GEMM1_SILU>(ma, mb, mb16, expert_off, E, K, N, FB, P, act, nullptr, status, st);
}

cudaError_t launch_pair_gemm2_scatter(int dtype, const void* act, int64_t P, const void* w2, int E, int K, int N,
                                      const int32_t* expert_off, const int32_t* sorted_pairs, void* y_slots,
                                      int* status, cudaStream_t st) {
  CUtensorMap ma, mb, mb16;
  const uint64_t a_dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)E};
  const uint64_t a_str[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
  const uint64_t b_dims[2] = {(uint64_t)N, (uint64_t)P};
  const uint64_t b_str[1] = {(uint64_t)N * 2};
  if (!make_kmajor_map(&ma, dtype, w2, 3, a_dims, a_str, 128)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mb, dtype, act, 2, b_dims, b_str, 128)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mb16, dtype, act, 2, b_dims, b_str, 16)) return cudaErrorInvalidValue;
  const int FB = (int)ceil_div(K, 256);
  if (dtype == MOE_DTYPE_BF16)
    return launch_pair_t<__nv_bfloat16, PAIR_GEMM2>(ma, mb, mb16, expert_off, E, N, K, FB, P, y_slots, sorted_pairs,
                                                    status, st);
  return launch_pair_t<__half, PAIR_GEMM2>(ma, mb, mb16, expert_off, E, N, K, FB, P, y_slots, sorted_pairs, status,
                                           st);
}

}  // namespace moe

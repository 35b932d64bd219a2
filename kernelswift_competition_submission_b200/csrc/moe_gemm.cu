// Grouped expert GEMMs on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One persistent, warp-specialised kernel template serves both expert GEMMs of
// fused_moe/v0/fused_moe.py:160-163:
//   GEMM1_SILU : act[r, n]  = silu(x_r . w1[e, n]) * (x_r . w1[e, N + n])     (:160-162)
//   GEMM2      : y[pair(r)] = act_r . w2[e]^T                                  (:163)
//   GEMM2_COMBINE: GEMM2, then the top-k weighted sum of :165-167 in the epilogue:
//               out[t] = sum_j topk_weights[t, j] * y[t * topk + j]
// Rows r come from the align stage: pairs grouped by expert e in m-blocks of
// 128 rows (block_start[e] .. block_start[e+1]).
//
// Tile = 128 rows x BN output columns, K consumed 64 elements (128 bytes) per
// pipeline stage:
//   warp 0      TMA producer: one elected lane loads the A box (128 x 64) and the
//               B box(es) (BN x 64) of each stage, 128-byte swizzle, completion
//               counted in bytes on the stage's `full` mbarrier.
//   warp 1      MMA issuer: one lane issues 4 x tcgen05.mma (M=128, N=BN, K=16)
//               per stage into a TMEM accumulator and commits the stage's
//               `empty` mbarrier; after the last stage of a tile it commits
//               `tmem_full` of that accumulator.
//   warp 2      TMEM allocator (2 accumulators x BN fp32 columns).
//   warps 4-7   epilogue: warp w reads TMEM lanes 32(w-4)..+31 (one row per
//               thread) with tcgen05.ld, applies SiLU*mul (GEMM1) or the
//               pair scatter (GEMM2), stores to global and releases the
//               accumulator, so the epilogue of tile i overlaps the MMAs of i+1.
// For GEMM1 the B tile stacks the gate rows [n0, n0+BN/2) over the up rows
// [N+n0, N+n0+BN/2) of the same expert, so gate and up of column n land in
// the same accumulator row and SiLU*mul needs no extra pass or weight copy.
//
// GEMM1_GATHER is GEMM1_SILU with the A tile gathered from the token rows instead of
// loaded from an expert-sorted copy: warps 2-3 (64 threads) copy, per stage, the 128-byte
// K slice of each of the tile's 128 rows (token sorted_pairs[r] / topk) with 16-byte
// cp.async into the 128-byte-swizzled layout the TMA would have written (chunk c of row r
// at r * 128 + ((c ^ (r & 7)) * 16)). Each thread keeps up to kGatherLag stages in flight;
// when a stage's copies are complete it fences them for the async proxy (the tensor core
// reads them) and arrives on the stage's `full` barrier, which also counts the TMA bytes
// of the B tile; it announces the oldest stage before it waits for a free one, so the
// MMAs never wait behind that wait. No row copy of the tokens is made anywhere.
//
// Tile order: expert-major, then n-block, then m-block fastest, so concurrently
// running CTAs share the expert's B tile through L2.
// All mbarrier waits are bounded (common.cuh); on a timeout every role stops,
// the producer waits (bounded) for its copies in flight, the MMA warp waits for
// its MMAs, and TMEM is freed before the CTA exits.
#include "common.cuh"
#include "moe_internal.h"


namespace moe {
namespace {

enum { MODE_GEMM1_SILU = 0, MODE_GEMM2 = 1, MODE_GEMM2_COMBINE = 2, MODE_GEMM1_GATHER = 3 };

// A rows of MODE_GEMM1_GATHER: row r of the expert-sorted order is token
// sorted_pairs[r] / topk of x (row pitch ld elements); padding rows (-1) read as zeros.
struct RowGather {
  const void* x;
  int64_t ld;
  int topk;
};

// Fused top-k combine of MODE_GEMM2_COMBINE. Every (token, n-block) has an arrival
// counter; after a warp has stored its 32 slot rows of one tile it counts each row's
// arrival, and the warp that brings a token's last valid slot of that n-block sums all
// of that token's slots over the n-block's columns (slot order, fp32 FMAs, one rounding:
// the arithmetic of combine_kernel, so the output bits do not depend on arrival order).
//
// Return mode (peer_base != nullptr; the expert-parallel layer over peer memory): row t of
// this launch is received row r = t % cap of source rank src = t / cap, and its sum goes
// straight into that rank's arena, back_x row me * cap + r (NVLink stores), instead of a
// local `out`. Every (row, n-block) segment stored counts once in src_done[src]; the warp
// that completes the source's own_counts[src] * NB segments raises back[me] = seq in that
// rank's arena (system-scope release after a system fence), and sources that sent no row
// get their flag at the start. With a failure already recorded in the status word the
// launch stores nothing into peers and raises no flag.
struct CombineArgs {
  const int32_t* ids;      // [M, topk] expert ids; slots outside [0, E) contribute nothing
  const float* weights;    // [M, topk]
  int32_t* arrivals;       // [M, NB], zero before the launch
  void* out;               // [M, n_out] (local mode)
  int topk;
  // return mode
  const int64_t* peer_base;   // [world] arena base of every rank
  const int32_t* own_counts;  // [world] rows each source sent this step (own arena)
  int32_t* src_done;          // [world] segments returned per source, zero before the launch
  int64_t back_off, flag_off; // byte offsets of back_x and of the back flags in an arena
  int64_t cap;                // rows per source region
  int me, world;
  uint32_t seq;
};

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr int kThreads = 256;
constexpr int kGatherThreads = 64;  // warps 2-3 in MODE_GEMM1_GATHER
constexpr int kGatherRows = kBlockM / (kGatherThreads / 8);  // rows per gather thread (16)
constexpr int kBK = 64;                    // K elements per stage (128 bytes of 16-bit data)
constexpr int kATileBytes = kBlockM * kBK * 2;

// Epilogue staging: each epilogue warp owns a [32 rows][64 columns] 16-bit tile
// with a 144-byte row pitch (128 + 16), so the per-row 16-byte writes and the
// per-segment 16-byte reads are both free of bank conflicts.
constexpr int kEpiPitch = 144;
constexpr int kEpiWarpBytes = 32 * kEpiPitch;

template <int BN, int STAGES>
struct SmemLayout {
  static constexpr int kBTileBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kEpiOffset = STAGES * kStageBytes;
  static constexpr int kBarOffset = kEpiOffset + 4 * kEpiWarpBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kBlockStartOffset = kMiscOffset + 16;
  static int bytes(int E) { return 1024 + kBlockStartOffset + 4 * (E + 1); }
};

__device__ __forceinline__ void decode_tile(const int* s_bs, int E, int NB, int tile, int& e, int& nb, int& mb) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_bs[mid] * NB <= tile) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int nblk = s_bs[lo + 1] - s_bs[lo];
  const int local = tile - s_bs[lo] * NB;
  nb = local / nblk;
  mb = s_bs[lo] + (local - nb * nblk);
}

// Arrival count and, for the rows whose arrival completes their token's n-block, the
// weighted slot sum (see CombineArgs). Called by a whole epilogue warp after its 32 rows
// (lane = row) of the tile's columns [nb * BN, nb * BN + BN) are stored to `slots`.
template <typename T, int BN>
__device__ __forceinline__ void combine_rows(const CombineArgs& cmb, const T* slots, int my_pair, int E, int NB,
                                             int nb, int n_out, int lane, bool remote_off) {
  const int topk = cmb.topk;
  __threadfence();  // this lane's slot stores are visible device-wide before its rows' arrivals count
  __syncwarp();
  int tok = 0;
  bool last = false;
  if (my_pair >= 0) {
    tok = my_pair / topk;
    const int32_t* tid = cmb.ids + (int64_t)tok * topk;
    int valid = 0;
    for (int j = 0; j < topk; ++j) {
      const int e = __ldg(tid + j);
      valid += (e >= 0 && e < E) ? 1 : 0;
    }
    last = atomicAdd(cmb.arrivals + (int64_t)tok * NB + nb, 1) == valid - 1;
  }
  uint32_t todo = __ballot_sync(0xffffffffu, last);
  if (todo == 0u) return;
  __threadfence();  // the other slots of these tokens were fenced before their arrivals
  T* out = static_cast<T*>(cmb.out);
  const int col = nb * BN + lane * 8;                  // this lane's 8 columns (BN = 128: lanes 16-31 idle)
  const bool col_ok = lane * 8 < BN && col < n_out;    // n_out % 64 == 0: a vector is whole or outside
  // kRows completed tokens per round with every slot load of the round in flight before the
  // first FMA (the slot rows come back from L2 / DRAM; one row at a time is latency-bound).
  // A slot outside [0, E) loads weight 0 and value 0: fma(0, 0, acc) == acc, so the sums are
  // the bits of combine_kernel, which skips such slots.
  constexpr int kRows = 4;
  while (todo) {
    int t[kRows];
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      t[q] = -1;
      if (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1u;
        t[q] = __shfl_sync(0xffffffffu, tok, src);
      }
    }
    float acc[kRows][8];
#pragma unroll
    for (int q = 0; q < kRows; ++q)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[q][i] = 0.f;
    for (int j0 = 0; j0 < topk; j0 += 8) {
      uint4 v[kRows][8];
      float wj[kRows][8];
#pragma unroll
      for (int q = 0; q < kRows; ++q) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u;
          const int e = (t[q] >= 0 && j < topk) ? __ldg(cmb.ids + (int64_t)t[q] * topk + j) : -1;
          const bool ok = col_ok && e >= 0 && e < E;
          wj[q][u] = ok ? __ldg(cmb.weights + (int64_t)t[q] * topk + j) : 0.f;
          v[q][u] = ok ? __ldcg(reinterpret_cast<const uint4*>(slots + ((int64_t)t[q] * topk + j) * n_out + col))
                       : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int q = 0; q < kRows; ++q) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t h[4] = {v[q][u].x, v[q][u].y, v[q][u].z, v[q][u].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = ElemTraits<T>::unpack2(h[i]);
            acc[q][2 * i] = fmaf(wj[q][u], f.x, acc[q][2 * i]);
            acc[q][2 * i + 1] = fmaf(wj[q][u], f.y, acc[q][2 * i + 1]);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      if (t[q] < 0 || !col_ok) continue;
      uint4 o;
      o.x = ElemTraits<T>::pack2(acc[q][0], acc[q][1]);
      o.y = ElemTraits<T>::pack2(acc[q][2], acc[q][3]);
      o.z = ElemTraits<T>::pack2(acc[q][4], acc[q][5]);
      o.w = ElemTraits<T>::pack2(acc[q][6], acc[q][7]);
      if (cmb.peer_base == nullptr) {
        *reinterpret_cast<uint4*>(out + (int64_t)t[q] * n_out + col) = o;
      } else if (!remote_off) {
        const int src = (int)(t[q] / cmb.cap);
        const int64_t r = t[q] - (int64_t)src * cmb.cap;
        T* dst = reinterpret_cast<T*>(reinterpret_cast<char*>(__ldg(cmb.peer_base + src)) + cmb.back_off);
        *reinterpret_cast<uint4*>(dst + ((int64_t)cmb.me * cmb.cap + r) * n_out + col) = o;
      }
    }
    if (cmb.peer_base != nullptr && !remote_off) {
      // these rows' segments of n-block nb are in their sources' arenas: count them, and
      // raise a source's flag when its last segment is in
      __threadfence_system();
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
          if (t[q] < 0) continue;
          const int src = (int)(t[q] / cmb.cap);
          const int want = __ldcg(cmb.own_counts + src) * NB;
          if (atomicAdd(cmb.src_done + src, 1) + 1 == want) {
            __threadfence_system();
            st_release_sys_u32(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(__ldg(cmb.peer_base + src)) +
                                                           cmb.flag_off) + cmb.me,
                               cmb.seq);
          }
        }
      }
      __syncwarp();
    }
  }
}

template <typename T, int MODE, int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
moe_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const int32_t* __restrict__ block_start, int E, int k_red, int n_out, int NB,
                T* __restrict__ out, const int32_t* __restrict__ sorted_pairs, int* status, CombineArgs cmb,
                RowGather gat) {
  using L = SmemLayout<BN, STAGES>;
  constexpr bool kGemm1 = MODE == MODE_GEMM1_SILU || MODE == MODE_GEMM1_GATHER;
  constexpr bool kGather = MODE == MODE_GEMM1_GATHER;
  constexpr int BH = kGemm1 ? BN / 2 : BN;   // rows per B box
  constexpr uint32_t kTmemCols = 2 * BN;
  constexpr uint32_t kIdesc = idesc_f16(kBlockM, BN, ElemTraits<T>::kFmt);
  // bytes the TMA delivers per stage: A and B, or B alone when the A rows are gathered
  constexpr uint32_t kStageTx = kGather ? (uint32_t)L::kBTileBytes : (uint32_t)L::kStageBytes;
  constexpr int kGatherLag = STAGES - 1;  // unannounced stages a gather thread keeps in flight

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tmem_full = bars + 2 * STAGES;
  uint64_t* tmem_empty = bars + 2 * STAGES + 2;
  uint64_t* mma_done = bars + 2 * STAGES + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);
  volatile int* s_remote_off = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 8);
  int* s_bs = reinterpret_cast<int*>(smem + L::kBlockStartOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i <= E; i += kThreads) s_bs[i] = __ldg(block_start + i);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], kGather ? 1 + kGatherThreads : 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tmem_full[a], 1); mbar_init(&tmem_empty[a], 128); }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    // return mode: a failure already recorded keeps this launch away from the peers' arenas
    *s_remote_off = (MODE == MODE_GEMM2_COMBINE && cmb.peer_base != nullptr && status != nullptr &&
                     *reinterpret_cast<volatile int*>(status) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  if constexpr (MODE == MODE_GEMM2_COMBINE) {
    if (cmb.peer_base != nullptr && blockIdx.x == 0 && (int)threadIdx.x < cmb.world &&
        (status == nullptr || *reinterpret_cast<volatile int*>(status) == 0) &&
        __ldcg(cmb.own_counts + threadIdx.x) == 0) {
      // a source that sent no row this step has nothing to wait for
      __threadfence_system();
      st_release_sys_u32(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(__ldg(cmb.peer_base + threadIdx.x)) +
                                                     cmb.flag_off) + cmb.me,
                         cmb.seq);
    }
  }
  if (warp == 0 && lane == 0) {
    if constexpr (!kGather) tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 2) { tmem_alloc(s_tmem, kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  const int total_tiles = s_bs[E] * NB;
  const int num_kb = (k_red + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        int e, nb, mb;
        decode_tile(s_bs, E, NB, tile, e, nb, mb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
          uint8_t* a_dst = smem + stage * L::kStageBytes;
          uint8_t* b_dst = a_dst + kATileBytes;
          mbar_arrive_expect_tx(&full[stage], kStageTx);
          if constexpr (!kGather) tma_load_2d(&map_a, &full[stage], a_dst, kb * kBK, mb * kBlockM);
          if constexpr (kGemm1) {
            tma_load_3d(&map_b, &full[stage], b_dst, kb * kBK, nb * BH, 2 * e);
            tma_load_3d(&map_b, &full[stage], b_dst + BH * kBK * 2, kb * kBK, nb * BH, 2 * e + 1);
          } else {
            tma_load_3d(&map_b, &full[stage], b_dst, kb * kBK, nb * BN, e);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // drain: wait (bounded, ignoring the abort flag) for the last copy issued into each stage
        for (int s = 0; s < STAGES; ++s)
          if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, nullptr);
      }
    }
  } else if (kGather && (warp == 2 || warp == 3)) {
    // ------------------------------------------------ A-row gather (cp.async)
    const int gt = threadIdx.x - 64;  // 0 .. kGatherThreads - 1
    const int c = gt & 7;             // 16-byte chunk of the row's 128-byte K slice
    const int rg = gt >> 3;           // rows rg, rg + 8, ..., rg + 120 (so r & 7 == rg)
    const uint32_t dst_off = (uint32_t)(rg * 128 + ((c ^ rg) << 4));
    const T* xb = static_cast<const T*>(gat.x);
    uint32_t issued = 0, announced = 0;  // k-iterations copied / arrived on `full`
    bool ok = true;
    int64_t row_off[kGatherRows];
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      int e, nb, mb;
      decode_tile(s_bs, E, NB, tile, e, nb, mb);
#pragma unroll
      for (int i = 0; i < kGatherRows; ++i) {
        const int pair = __ldg(sorted_pairs + (int64_t)mb * kBlockM + rg + 8 * i);
        row_off[i] = pair >= 0 ? (int64_t)(pair / gat.topk) * gat.ld + c * 8 : -1;
      }
      for (int kb = 0; kb < num_kb; ++kb) {
        // announce the oldest stage in flight as soon as it has landed, before waiting for
        // the next free stage: the MMAs of a stage must not wait for that wait
        if (issued - announced >= (uint32_t)kGatherLag) {
          cp_async_wait_group<kGatherLag - 1>();
          fence_proxy_async_smem();
          mbar_arrive(&full[announced % STAGES]);
          ++announced;
        }
        const int stage = (int)(issued % STAGES);
        const uint32_t phase = (issued / STAGES) & 1u;
        if (!mbar_wait(&empty[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
        const uint32_t a_dst = smem_u32(smem + stage * L::kStageBytes) + dst_off;
#pragma unroll
        for (int i = 0; i < kGatherRows; ++i) {
          const bool live = row_off[i] >= 0;
          cp_async_16(a_dst + i * 1024, live ? xb + row_off[i] + kb * kBK : xb, live ? 16u : 0u);
        }
        cp_async_commit();
        ++issued;
      }
    }
    // every copy lands before the stages are announced (and before the CTA can exit)
    cp_async_wait_all();
    fence_proxy_async_smem();
    for (; announced < issued; ++announced) mbar_arrive(&full[announced % STAGES]);
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, status, s_abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* a_src = smem + stage * L::kStageBytes;
          const uint64_t a_desc = smem_desc_sw128(a_src);
          const uint64_t b_desc = smem_desc_sw128(a_src + kATileBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes along K inside the 128-byte swizzled row = +2 in the address field
            umma_f16(d_tmem, a_desc + 2 * k, b_desc + 2 * k, kIdesc, (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // all MMAs issued by this thread complete before TMEM is freed
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, nullptr);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ epilogue
    // Each warp owns TMEM lanes 32*ew .. +31 (= tile rows). Per group of 64 output
    // columns: tcgen05.ld two 32-column chunks (one row per thread), convert, stage
    // in the warp's shared tile, then store whole 128-byte row segments: lane l
    // writes 16-byte chunk (l & 7) of row 4*i + (l >> 3), so one warp store covers
    // four full segments instead of 32 half-sectors.
    const int ew = warp - 4;
    uint8_t* stage = smem + L::kEpiOffset + ew * kEpiWarpBytes;
    const int st_r = lane >> 3, st_c = lane & 7;
    constexpr int kGroups = (kGemm1 ? BH : BN) / 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int e, nb, mb;
      decode_tile(s_bs, E, NB, tile, e, nb, mb);
      // warp-uniform decision: tcgen05.ld below is .sync.aligned
      if (!__all_sync(0xffffffffu, mbar_wait(&tmem_full[acc], acc_phase, status, s_abort))) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
      const int64_t row0 = (int64_t)mb * kBlockM + ew * 32;  // first tile row of this warp
      int my_pair = 0;
      if constexpr (!kGemm1) my_pair = __ldg(sorted_pairs + row0 + lane);
#pragma unroll 1
      for (int g = 0; g < kGroups; ++g) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = 2 * g + h;  // 32-column chunk
          uint32_t packed[16];
          if constexpr (kGemm1) {
            uint32_t gt[32], up[32];
            tmem_ld32(t_row + c * 32, gt);
            tmem_ld32(t_row + BH + c * 32, up);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float g0 = __uint_as_float(gt[2 * i]), g1 = __uint_as_float(gt[2 * i + 1]);
              const float u0 = __uint_as_float(up[2 * i]), u1 = __uint_as_float(up[2 * i + 1]);
              packed[i] = ElemTraits<T>::pack2(g0 / (1.0f + __expf(-g0)) * u0, g1 / (1.0f + __expf(-g1)) * u1);
            }
          } else {
            uint32_t v[32];
            tmem_ld32(t_row + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i)
              packed[i] = ElemTraits<T>::pack2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          }
          uint4* srow = reinterpret_cast<uint4*>(stage + lane * kEpiPitch + h * 64);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            srow[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
        }
        if (g == kGroups - 1) {
          // accumulator fully read: release it to the MMA warp before the last stores
          tc_fence_before();
          mbar_arrive(&tmem_empty[acc]);
        }
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int r = 4 * it + st_r;
          const uint4 val = *reinterpret_cast<const uint4*>(stage + r * kEpiPitch + st_c * 16);
          if constexpr (kGemm1) {
            T* dst = out + (row0 + r) * (int64_t)n_out + (int64_t)nb * BH + g * 64 + st_c * 8;
            *reinterpret_cast<uint4*>(dst) = val;
          } else {
            const int pair = __shfl_sync(0xffffffffu, my_pair, r);
            const int col = nb * BN + g * 64;
            if (pair >= 0 && col < n_out)
              *reinterpret_cast<uint4*>(out + (int64_t)pair * n_out + col + st_c * 8) = val;
          }
        }
        __syncwarp();
      }
      if constexpr (MODE == MODE_GEMM2_COMBINE)
        combine_rows<T, BN>(cmb, out, my_pair, E, NB, nb, n_out, lane, *s_remote_off != 0);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
constexpr int kStages = 4;

template <typename T, int MODE, int BN>
cudaError_t launch_gemm_t(const CUtensorMap& ma, const CUtensorMap& mb, const int32_t* block_start, int E, int k_red,
                          int n_out, int NB, int64_t rows_cap, void* out, const int32_t* sorted_pairs, int* status,
                          int max_ctas, cudaStream_t st, const CombineArgs& cmb = CombineArgs{},
                          const RowGather& gat = RowGather{}) {
  using L = SmemLayout<BN, kStages>;
  auto kern = moe_gemm_kernel<T, MODE, BN, kStages>;
  const int smem = L::bytes(E);
  cudaError_t err = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
  if (err != cudaSuccess) return err;
  const int64_t tiles_cap = (rows_cap / kBlockM) * NB;
  // persistent grid: one CTA per SM, or fewer when the caller keeps SMs free for
  // concurrent work (e.g. collectives overlapping the GEMM)
  const int ctas = (max_ctas > 0 && max_ctas < num_sms()) ? max_ctas : num_sms();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas, tiles_cap));
  kern<<<grid, kThreads, smem, st>>>(ma, mb, block_start, E, k_red, n_out, NB, static_cast<T*>(out), sorted_pairs,
                                     status, cmb, gat);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm1_silu(int dtype, const void* x_sorted, int64_t rows_cap, const void* w1, int E, int K, int N,
                              const int32_t* block_start, void* act, int* status, int max_ctas, cudaStream_t st) {
  const int BN = (N % 128 == 0) ? 256 : 128;
  const int BH = BN / 2;
  CUtensorMap ma, mbm;
  const uint64_t a_dims[2] = {(uint64_t)K, (uint64_t)rows_cap};
  const uint64_t a_str[1] = {(uint64_t)K * 2};
  const uint64_t b_dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)2 * E};
  const uint64_t b_str[2] = {(uint64_t)K * 2, (uint64_t)N * K * 2};
  if (!make_kmajor_map(&ma, dtype, x_sorted, 2, a_dims, a_str, kBlockM)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mbm, dtype, w1, 3, b_dims, b_str, (uint32_t)BH)) return cudaErrorInvalidValue;
  const int NB = N / BH;
  if (dtype == MOE_DTYPE_BF16) {
    if (BN == 256)
      return launch_gemm_t<__nv_bfloat16, MODE_GEMM1_SILU, 256>(ma, mbm, block_start, E, K, N, NB, rows_cap, act,
                                                                nullptr, status, max_ctas, st);
    return launch_gemm_t<__nv_bfloat16, MODE_GEMM1_SILU, 128>(ma, mbm, block_start, E, K, N, NB, rows_cap, act,
                                                              nullptr, status, max_ctas, st);
  }
  if (BN == 256)
    return launch_gemm_t<__half, MODE_GEMM1_SILU, 256>(ma, mbm, block_start, E, K, N, NB, rows_cap, act, nullptr,
                                                       status, max_ctas, st);
  return launch_gemm_t<__half, MODE_GEMM1_SILU, 128>(ma, mbm, block_start, E, K, N, NB, rows_cap, act, nullptr,
                                                     status, max_ctas, st);
}

int gemm2_block_n(int K) { return (K >= 256) ? 256 : 128; }

namespace {

// GEMM2 (slot rows) or GEMM2_COMBINE (slot rows + fused top-k sum into cmb.out).
template <int MODE>
cudaError_t launch_gemm2_mode(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                              const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots, int* status,
                              int max_ctas, cudaStream_t st, const CombineArgs& cmb) {
  const int BN = gemm2_block_n(K);
  CUtensorMap ma, mbm;
  const uint64_t a_dims[2] = {(uint64_t)N, (uint64_t)rows_cap};
  const uint64_t a_str[1] = {(uint64_t)N * 2};
  const uint64_t b_dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)E};
  const uint64_t b_str[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
  if (!make_kmajor_map(&ma, dtype, act, 2, a_dims, a_str, kBlockM)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mbm, dtype, w2, 3, b_dims, b_str, (uint32_t)BN)) return cudaErrorInvalidValue;
  const int NB = (int)ceil_div(K, BN);
  if (dtype == MOE_DTYPE_BF16) {
    if (BN == 256)
      return launch_gemm_t<__nv_bfloat16, MODE, 256>(ma, mbm, block_start, E, N, K, NB, rows_cap, y_slots,
                                                     sorted_pairs, status, max_ctas, st, cmb);
    return launch_gemm_t<__nv_bfloat16, MODE, 128>(ma, mbm, block_start, E, N, K, NB, rows_cap, y_slots,
                                                   sorted_pairs, status, max_ctas, st, cmb);
  }
  if (BN == 256)
    return launch_gemm_t<__half, MODE, 256>(ma, mbm, block_start, E, N, K, NB, rows_cap, y_slots, sorted_pairs,
                                            status, max_ctas, st, cmb);
  return launch_gemm_t<__half, MODE, 128>(ma, mbm, block_start, E, N, K, NB, rows_cap, y_slots, sorted_pairs,
                                          status, max_ctas, st, cmb);
}

}  // namespace

cudaError_t launch_gemm1_gather(int dtype, const void* x, int64_t x_ld, int topk, const int32_t* sorted_pairs,
                               int64_t rows_cap, const void* w1, int E, int K, int N, const int32_t* block_start,
                               void* act, int* status, int max_ctas, cudaStream_t st) {
  const int BN = (N % 128 == 0) ? 256 : 128;
  const int BH = BN / 2;
  CUtensorMap mbm;
  const uint64_t b_dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)2 * E};
  const uint64_t b_str[2] = {(uint64_t)K * 2, (uint64_t)N * K * 2};
  if (!make_kmajor_map(&mbm, dtype, w1, 3, b_dims, b_str, (uint32_t)BH)) return cudaErrorInvalidValue;
  const int NB = N / BH;
  const RowGather gat{x, x_ld, topk};
  // the A map is unused in this mode (the rows are gathered); the B map fills its slot
  if (dtype == MOE_DTYPE_BF16) {
    if (BN == 256)
      return launch_gemm_t<__nv_bfloat16, MODE_GEMM1_GATHER, 256>(mbm, mbm, block_start, E, K, N, NB, rows_cap, act,
                                                                  sorted_pairs, status, max_ctas, st, CombineArgs{},
                                                                  gat);
    return launch_gemm_t<__nv_bfloat16, MODE_GEMM1_GATHER, 128>(mbm, mbm, block_start, E, K, N, NB, rows_cap, act,
                                                                sorted_pairs, status, max_ctas, st, CombineArgs{}, gat);
  }
  if (BN == 256)
    return launch_gemm_t<__half, MODE_GEMM1_GATHER, 256>(mbm, mbm, block_start, E, K, N, NB, rows_cap, act,
                                                         sorted_pairs, status, max_ctas, st, CombineArgs{}, gat);
  return launch_gemm_t<__half, MODE_GEMM1_GATHER, 128>(mbm, mbm, block_start, E, K, N, NB, rows_cap, act, sorted_pairs,
                                                       status, max_ctas, st, CombineArgs{}, gat);
}

cudaError_t launch_gemm2_scatter(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                                 const int32_t* block_start, const int32_t* sorted_pairs, int64_t num_pairs,
                                 void* y_slots, int* status, int max_ctas, cudaStream_t st) {
  (void)num_pairs;
  return launch_gemm2_mode<MODE_GEMM2>(dtype, act, rows_cap, w2, E, K, N, block_start, sorted_pairs, y_slots, status,
                                       max_ctas, st, CombineArgs{});
}

cudaError_t launch_gemm2_return(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                                const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots,
                                const float* recv_w, const int32_t* recv_id, int topk, int32_t* arrivals,
                                const int64_t* peer_base, const int32_t* own_counts, int32_t* src_done,
                                int64_t back_off, int64_t flag_off, int64_t cap, int me, int world, uint32_t seq,
                                int* status, int max_ctas, cudaStream_t st) {
  CombineArgs cmb{recv_id, recv_w, arrivals, nullptr, topk};
  cmb.peer_base = peer_base;
  cmb.own_counts = own_counts;
  cmb.src_done = src_done;
  cmb.back_off = back_off;
  cmb.flag_off = flag_off;
  cmb.cap = cap;
  cmb.me = me;
  cmb.world = world;
  cmb.seq = seq;
  return launch_gemm2_mode<MODE_GEMM2_COMBINE>(dtype, act, rows_cap, w2, E, K, N, block_start, sorted_pairs, y_slots,
                                               status, max_ctas, st, cmb);
}

cudaError_t launch_gemm2_combine(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                                 const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots,
                                 const float* topk_weights, const int32_t* topk_ids, int topk, int32_t* arrivals,
                                 void* out, int* status, int max_ctas, cudaStream_t st) {
  CombineArgs cmb{topk_ids, topk_weights, arrivals, out, topk};
  return launch_gemm2_mode<MODE_GEMM2_COMBINE>(dtype, act, rows_cap, w2, E, K, N, block_start, sorted_pairs, y_slots,
                                               status, max_ctas, st, cmb);
}

}  // namespace moe

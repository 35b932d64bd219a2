// Grouped expert GEMMs for the FP8 w8a8 configuration (DeepSeek-V3 recipe:
// e4m3 weights with an fp32 scale per 128 x 128 block, e4m3 activations with an
// fp32 scale per token per 128 channels). The math is the expert path of
// fused_moe/v0/fused_moe.py:160-163 on dequantised operands.
//
// Why the MMA runs in bf16: tcgen05's block-scaled MMA kinds take power-of-two
// (ue8m0) scales per 32 elements; fp32 scales per 128 x 128 block cannot be
// folded into them exactly. Instead the e4m3 tiles stream from HBM at 1 byte per
// element (half the bf16 bytes: the layer is HBM-bound on the weight stream at
// the decode sizes this configuration targets), and converter warps turn each
// stage into the bf16 swizzled tiles of the same tcgen05 pipeline:
//
//   warp 0      TMA producer: e4m3 A box (128 rows x 64 B) and B box(es)
//               (BN rows x 64 B) per 64-wide K step, into `fp8` stages.
//   warps 2,3,8-11  converters (warp 2 after allocating TMEM): e4m3 -> fp32 * scale -> bf16, in the
//               128-byte-swizzled K-major layout the MMA descriptors expect
//               (16-byte chunk c of row r at chunk c ^ (r & 7)); then
//               fence.proxy.async so the tensor core sees the writes.
//   warp 1      MMA issuer (kind::f16, bf16 in, fp32 accumulate in TMEM).
//   warp 2      TMEM allocator (2 accumulators x BN columns).
//   warps 4-7   epilogue. GEMM1: two TMEM passes per row (amax of the row's 128
//               SiLU*mul outputs, then quantise with scale = amax / 448) ->
//               e4m3 act row + its scale, the A operand of GEMM2. GEMM2: bf16
//               rows of the pair slots, as in the bf16 path.
// Rows come from the align stage (pairs grouped by expert, 128-row m-blocks).
// All mbarrier waits are bounded; named barriers keep each role group's
// decisions uniform so no group can be left waiting on a barrier.
#include "common.cuh"
#include "moe_internal.h"

#include <cuda_fp8.h>

namespace moe {
namespace {

enum { F8_GEMM1 = 0, F8_GEMM2 = 1 };

constexpr int kF8Threads = 384;
constexpr int kF8BK = 64;                      // K elements per stage
constexpr int kS8 = 4;                         // e4m3 stages
constexpr int kS16 = 2;                        // bf16 stages
constexpr int kA8Bytes = kBlockM * kF8BK;      // 8 KB
constexpr int kA16Bytes = kBlockM * kF8BK * 2; // 16 KB
constexpr int kEpiPitchF8 = 144;
constexpr int kEpiWarpBytesF8 = 32 * kEpiPitchF8;

template <int BN>
struct F8Layout {
  static constexpr int kB8Bytes = BN * kF8BK;
  static constexpr int kStage8 = kA8Bytes + kB8Bytes;
  static constexpr int kStage16 = kA16Bytes + BN * kF8BK * 2;
  static constexpr int kOff8 = 0;
  static constexpr int kOff16 = kS8 * kStage8;                 // multiple of 1024
  static constexpr int kEpiOffset = kOff16 + kS16 * kStage16;
  static constexpr int kAScaleOffset = kEpiOffset + 4 * kEpiWarpBytesF8;  // [2][128] fp32: A row scales, 2 K blocks
  static constexpr int kBScaleOffset = kAScaleOffset + 2 * 128 * 4;       // [2][128] fp32: B block scales of a tile
  static constexpr int kBarOffset = kBScaleOffset + 2 * 128 * 4;
  static constexpr int kNumBars = 2 * kS8 + 2 * kS16 + 5;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kBlockStartOffset = kMiscOffset + 16;
  static int bytes(int E) { return 1024 + kBlockStartOffset + 4 * (E + 1) + 4 * E; }
};

__device__ __forceinline__ void decode_tile_f8(const int* s_bs, int E, int NB, int tile, int& e, int& nb, int& mb) {
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

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 8 e4m3 bytes (one 64-bit word) * scale -> 8 bf16 (16 bytes)
__device__ __forceinline__ uint4 dequant8(uint2 raw, float sc) {
  const uint32_t w[2] = {raw.x, raw.y};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((w[i] >> (16 * h)) & 0xFFFFu);
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
      __nv_bfloat162 b = __floats2bfloat162_rn(f.x * sc, f.y * sc);
      o[2 * i + h] = *reinterpret_cast<uint32_t*>(&b);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint32_t quant4(const float* v, float sc) {
  uint32_t p = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) p |= (uint32_t)__nv_cvt_float_to_fp8(v[i] / sc, __NV_SATFINITE, __NV_E4M3) << (8 * i);
  return p;
}

template <int MODE, int BN>
__global__ void __launch_bounds__(kF8Threads, 1)
moe_gemm_fp8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const float* __restrict__ a_scale, int a_scale_cols, const float* __restrict__ b_scale,
                    const int32_t* __restrict__ block_start, const int32_t* __restrict__ expert_counts, int E,
                    int k_red, int n_out, int NB, void* __restrict__ out, float* __restrict__ out_scale,
                    const int32_t* __restrict__ sorted_pairs, int* status) {
  using L = F8Layout<BN>;
  constexpr int BH = (MODE == F8_GEMM1) ? BN / 2 : BN;
  constexpr uint32_t kTmemCols = 2 * BN;
  constexpr uint32_t kIdesc = idesc_f16(kBlockM, BN, 1);
  constexpr uint32_t kStageTx = L::kStage8;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full8 = bars;
  uint64_t* empty8 = bars + kS8;
  uint64_t* full16 = bars + 2 * kS8;
  uint64_t* empty16 = full16 + kS16;
  uint64_t* tmem_full = full16 + 2 * kS16;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_done = tmem_full + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);
  int* s_bs = reinterpret_cast<int*>(smem + L::kBlockStartOffset);
  int* s_cnt = s_bs + (E + 1);  // pairs per expert

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i <= E; i += kF8Threads) s_bs[i] = __ldg(block_start + i);
  for (int i = threadIdx.x; i < E; i += kF8Threads) s_cnt[i] = __ldg(expert_counts + i);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kS8; ++s) { mbar_init(&full8[s], 1); mbar_init(&empty8[s], 1); }
    for (int s = 0; s < kS16; ++s) { mbar_init(&full16[s], 1); mbar_init(&empty16[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tmem_full[a], 1); mbar_init(&tmem_empty[a], 128); }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&map_a); tma_prefetch_desc(&map_b); }
  if (warp == 2) { tmem_alloc(s_tmem, kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_tiles = s_bs[E] * NB;
  const int num_kb = (k_red + kF8BK - 1) / kF8BK;
  const int kblocks128 = (k_red + 127) / 128;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (e4m3 stages)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        int e, nb, mb;
        decode_tile_f8(s_bs, E, NB, tile, e, nb, mb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty8[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
          uint8_t* a_dst = smem + L::kOff8 + stage * L::kStage8;
          uint8_t* b_dst = a_dst + kA8Bytes;
          mbar_arrive_expect_tx(&full8[stage], kStageTx);
          tma_load_2d(&map_a, &full8[stage], a_dst, kb * kF8BK, mb * kBlockM);
          if constexpr (MODE == F8_GEMM1) {
            tma_load_3d(&map_b, &full8[stage], b_dst, kb * kF8BK, nb * BH, 2 * e);
            tma_load_3d(&map_b, &full8[stage], b_dst + BH * kF8BK, kb * kF8BK, nb * BH, 2 * e + 1);
          } else {
            tma_load_3d(&map_b, &full8[stage], b_dst, kb * kF8BK, nb * BN, e);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kS8) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        for (int s = 0; s < kS8; ++s)
          if ((issued_mask >> s) & 1u) mbar_wait(&full8[s], (issued_parity >> s) & 1u, nullptr, nullptr);
      }
    }
  } else if (warp >= 8 || warp == 3 || (warp == 2)) {
    // ------------------------------------------------ converters (e4m3 -> bf16 swizzled), 6 warps
    // Warps 2 (after the TMEM allocation) and 3 join warps 8-11: 192 threads.
    const int ct = (warp < 8) ? (warp - 2) * 32 + lane : 64 + (threadIdx.x - 256);
    constexpr int kNT = 192;
    float* s_ascale = reinterpret_cast<float*>(smem + L::kAScaleOffset);  // [kq & 1][row]
    float* s_bscale = reinterpret_cast<float*>(smem + L::kBScaleOffset);  // [half][kq], kblocks128 <= 128
    int s8 = 0, s16 = 0;
    uint32_t p8 = 0, p16 = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int e, nb, mb;
      decode_tile_f8(s_bs, E, NB, tile, e, nb, mb);
      // rows of this m-block that hold pairs; the rest are padding whose results are
      // never stored, so their A rows are not converted (the MMA sees stale values there)
      const int valid = min(kBlockM, max(0, s_cnt[e] - (mb - s_bs[e]) * kBlockM));
      // the tile's weight-block scales (two 128-row blocks of B, every K block) and the
      // first K block's row scales, staged before the first stage is converted
      const float* bs0;
      const float* bs1;
      if constexpr (MODE == F8_GEMM1) {
        const int nrb = 2 * (n_out / 128);  // w1 row blocks per expert: gate blocks, then up blocks
        bs0 = b_scale + ((int64_t)e * nrb + nb) * kblocks128;
        bs1 = b_scale + ((int64_t)e * nrb + n_out / 128 + nb) * kblocks128;
      } else {
        const int nrb = (n_out + 127) / 128;
        const int rb0 = nb * (BN / 128);
        bs0 = b_scale + ((int64_t)e * nrb + rb0) * kblocks128;
        bs1 = (BN == 256 && rb0 + 1 < nrb) ? bs0 + kblocks128 : bs0;
      }
      for (int i = ct; i < 2 * kblocks128; i += kNT) s_bscale[i] = __ldg(i < kblocks128 ? bs0 + i : bs1 + (i - kblocks128));
      const float* arow = a_scale + ((int64_t)mb * kBlockM + ct) * a_scale_cols;
      if (ct < valid) s_ascale[ct] = __ldg(arow);
      float a_next = (ct < valid && kblocks128 > 1) ? __ldg(arow + 1) : 0.f;  // prefetch of K block 1
      named_bar_sync(2, kNT);
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int kq = kb * kF8BK / 128;  // 128-wide scale block along K
        const bool got = mbar_wait(&full8[s8], p8, status, s_abort) && mbar_wait(&empty16[s16], p16 ^ 1, status, s_abort);
        if (!named_bar_and(2, kNT, got)) { ok = false; break; }
        if (kb > 0 && (kb * kF8BK) % 128 == 0) {
          // new K block: publish the prefetched row scales, prefetch the next block's
          if (ct < valid) s_ascale[(kq & 1) * 128 + ct] = a_next;
          a_next = (ct < valid && kq + 1 < kblocks128) ? __ldg(arow + kq + 1) : 0.f;
          named_bar_sync(2, kNT);
        }
        const float bsc0 = s_bscale[kq];
        const float bsc1 = s_bscale[kblocks128 + kq];
        const float* ascale = s_ascale + (kq & 1) * 128;
        const uint8_t* a8 = smem + L::kOff8 + s8 * L::kStage8;
        const uint8_t* b8 = a8 + kA8Bytes;
        uint8_t* a16 = smem + L::kOff16 + s16 * L::kStage16;
        uint8_t* b16 = a16 + kA16Bytes;
        const int c = ct & 7;  // this thread's 16-byte chunk column (kNT is a multiple of 8)
#pragma unroll 4
        for (int row = ct >> 3; row < BN; row += kNT / 8) {
          const uint2 raw = *reinterpret_cast<const uint2*>(b8 + row * kF8BK + c * 8);
          *reinterpret_cast<uint4*>(b16 + row * 128 + ((c ^ (row & 7)) << 4)) = dequant8(raw, row < 128 ? bsc0 : bsc1);
        }
#pragma unroll 4
        for (int row = ct >> 3; row < valid; row += kNT / 8) {
          const uint2 raw = *reinterpret_cast<const uint2*>(a8 + row * kF8BK + c * 8);
          *reinterpret_cast<uint4*>(a16 + row * 128 + ((c ^ (row & 7)) << 4)) = dequant8(raw, ascale[row]);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> tensor-core (async proxy) reads
        named_bar_sync(2, kNT);
        if (ct == 0) {
          mbar_arrive(&full16[s16]);
          mbar_arrive(&empty8[s8]);
        }
        if (++s8 == kS8) { s8 = 0; p8 ^= 1; }
        if (++s16 == kS16) { s16 = 0; p16 ^= 1; }
      }
      if (!ok) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer (bf16 stages)
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
          if (!mbar_wait(&full16[stage], phase, status, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* a_src = smem + L::kOff16 + stage * L::kStage16;
          const uint64_t a_desc = smem_desc_sw128(a_src);
          const uint64_t b_desc = smem_desc_sw128(a_src + kA16Bytes);
#pragma unroll
          for (int k = 0; k < kF8BK / 16; ++k)
            umma_f16(d_tmem, a_desc + 2 * k, b_desc + 2 * k, kIdesc, (kb | k) != 0);
          umma_commit(&empty16[stage]);
          if (++stage == kS16) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, nullptr);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ epilogue
    const int ew = warp - 4;
    uint8_t* stage = smem + L::kEpiOffset + ew * kEpiWarpBytesF8;
    const int st_r = lane >> 3, st_c = lane & 7;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int e, nb, mb;
      decode_tile_f8(s_bs, E, NB, tile, e, nb, mb);
      if (!__all_sync(0xffffffffu, mbar_wait(&tmem_full[acc], acc_phase, status, s_abort))) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
      const int64_t row0 = (int64_t)mb * kBlockM + ew * 32;
      if constexpr (MODE == F8_GEMM1) {
        // pass 1: amax of this row's BH (= 128) SiLU*mul outputs
        float amax = 0.f;
#pragma unroll 1
        for (int c = 0; c < BH / 32; ++c) {
          uint32_t gt[32], up[32];
          tmem_ld32(t_row + c * 32, gt);
          tmem_ld32(t_row + BH + c * 32, up);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float g = __uint_as_float(gt[i]);
            amax = fmaxf(amax, fabsf(g / (1.0f + __expf(-g)) * __uint_as_float(up[i])));
          }
        }
        const float sc = amax > 0.f ? amax / 448.0f : 1.0f;
        // pass 2: quantise to e4m3 (32 values -> 32 bytes per chunk) into the staging row
#pragma unroll 1
        for (int c = 0; c < BH / 32; ++c) {
          uint32_t gt[32], up[32];
          tmem_ld32(t_row + c * 32, gt);
          tmem_ld32(t_row + BH + c * 32, up);
          tmem_wait_ld();
          uint32_t packed[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float a[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float g = __uint_as_float(gt[4 * i + j]);
              a[j] = g / (1.0f + __expf(-g)) * __uint_as_float(up[4 * i + j]);
            }
            packed[i] = quant4(a, sc);
          }
          uint4* srow = reinterpret_cast<uint4*>(stage + lane * kEpiPitchF8 + c * 32);
          srow[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          srow[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
        tc_fence_before();
        mbar_arrive(&tmem_empty[acc]);
        // scale of this row's 128-column block of act
        out_scale[(row0 + lane) * (int64_t)(n_out / 128) + nb] = sc;
        __syncwarp();
        uint8_t* act = static_cast<uint8_t*>(out);
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int r = 4 * it + st_r;
          const uint4 val = *reinterpret_cast<const uint4*>(stage + r * kEpiPitchF8 + st_c * 16);
          *reinterpret_cast<uint4*>(act + (row0 + r) * (int64_t)n_out + (int64_t)nb * BH + st_c * 16) = val;
        }
        __syncwarp();
      } else {
        int my_pair = __ldg(sorted_pairs + row0 + lane);
        __nv_bfloat16* y = static_cast<__nv_bfloat16*>(out);
#pragma unroll 1
        for (int g = 0; g < BN / 64; ++g) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t v[32];
            tmem_ld32(t_row + (2 * g + h) * 32, v);
            tmem_wait_ld();
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
              packed[i] = *reinterpret_cast<uint32_t*>(&b);
            }
            uint4* srow = reinterpret_cast<uint4*>(stage + lane * kEpiPitchF8 + h * 64);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              srow[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
          }
          if (g == BN / 64 - 1) {
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
          }
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int r = 4 * it + st_r;
            const uint4 val = *reinterpret_cast<const uint4*>(stage + r * kEpiPitchF8 + st_c * 16);
            const int pair = __shfl_sync(0xffffffffu, my_pair, r);
            const int col = nb * BN + g * 64;
            if (pair >= 0 && col < n_out)
              *reinterpret_cast<uint4*>(y + (int64_t)pair * n_out + col + st_c * 8) = val;
          }
          __syncwarp();
        }
      }
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

// Gather of whole rows into expert-sorted order: dst[r] = src[sorted_pairs[r] / topk]
// for the rows the align stage filled (r < block_start[E] * 128, pair >= 0).
__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint8_t* __restrict__ src, int64_t row_bytes, const int32_t* __restrict__ sorted_pairs,
                   const int32_t* __restrict__ block_start, int E, int topk, int64_t cap, uint8_t* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= cap || r >= (int64_t)__ldg(block_start + E) * kBlockM) return;
  const int pair = __ldg(sorted_pairs + r);
  if (pair < 0) return;
  const int64_t t = pair / topk;
  if ((row_bytes & 15) == 0) {
    const uint4* s = reinterpret_cast<const uint4*>(src + t * row_bytes);
    uint4* d = reinterpret_cast<uint4*>(dst + r * row_bytes);
    for (int64_t v = lane; v < row_bytes / 16; v += 32) d[v] = __ldg(s + v);
  } else {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src + t * row_bytes);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst + r * row_bytes);
    for (int64_t v = lane; v < row_bytes / 4; v += 32) d[v] = __ldg(s + v);
  }
}

template <int MODE, int BN>
cudaError_t launch_f8_t(const CUtensorMap& ma, const CUtensorMap& mb, const float* a_scale, int a_scale_cols,
                        const float* b_scale, const int32_t* block_start, const int32_t* expert_counts, int E,
                        int k_red, int n_out, int NB, int64_t rows_cap, void* out, float* out_scale,
                        const int32_t* sorted_pairs, int* status, cudaStream_t st) {
  using L = F8Layout<BN>;
  auto kern = moe_gemm_fp8_kernel<MODE, BN>;
  const int smem = L::bytes(E);
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  const int64_t tiles_cap = (rows_cap / kBlockM) * NB;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), tiles_cap));
  kern<<<grid, kF8Threads, smem, st>>>(ma, mb, a_scale, a_scale_cols, b_scale, block_start, expert_counts, E, k_red,
                                       n_out, NB, out, out_scale, sorted_pairs, status);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gather_rows(const void* src, int64_t row_bytes, const int32_t* sorted_pairs,
                               const int32_t* block_start, int E, int topk, int64_t cap, void* dst, cudaStream_t st) {
  if (cap == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)ceil_div(cap * 32, 256);
  gather_rows_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint8_t*>(src), row_bytes, sorted_pairs, block_start,
                                             E, topk, cap, static_cast<uint8_t*>(dst));
  return cudaGetLastError();
}

cudaError_t launch_fp8_gemm1(const void* xq_sorted, const float* xs_sorted, int64_t rows_cap, const void* w1q,
                             const float* w1s, int E, int K, int N, const int32_t* block_start,
                             const int32_t* expert_counts, void* actq, float* acts, int* status, cudaStream_t st) {
  CUtensorMap ma, mbm;
  const uint64_t a_dims[2] = {(uint64_t)K, (uint64_t)rows_cap};
  const uint64_t a_str[1] = {(uint64_t)K};
  const uint64_t b_dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)2 * E};
  const uint64_t b_str[2] = {(uint64_t)K, (uint64_t)N * K};
  if (!make_fp8_map(&ma, xq_sorted, 2, a_dims, a_str, kBlockM)) return cudaErrorInvalidValue;
  if (!make_fp8_map(&mbm, w1q, 3, b_dims, b_str, 128)) return cudaErrorInvalidValue;
  return launch_f8_t<F8_GEMM1, 256>(ma, mbm, xs_sorted, K / 128, w1s, block_start, expert_counts, E, K, N, N / 128,
                                    rows_cap, actq, acts, nullptr, status, st);
}

cudaError_t launch_fp8_gemm2(const void* actq, const float* acts, int64_t rows_cap, const void* w2q, const float* w2s,
                             int E, int K, int N, const int32_t* block_start, const int32_t* expert_counts,
                             const int32_t* sorted_pairs, void* y_slots, int* status, cudaStream_t st) {
  CUtensorMap ma, mbm;
  const uint64_t a_dims[2] = {(uint64_t)N, (uint64_t)rows_cap};
  const uint64_t a_str[1] = {(uint64_t)N};
  const uint64_t b_dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)E};
  const uint64_t b_str[2] = {(uint64_t)N, (uint64_t)K * N};
  if (!make_fp8_map(&ma, actq, 2, a_dims, a_str, kBlockM)) return cudaErrorInvalidValue;
  if (K >= 256) {
    if (!make_fp8_map(&mbm, w2q, 3, b_dims, b_str, 256)) return cudaErrorInvalidValue;
    return launch_f8_t<F8_GEMM2, 256>(ma, mbm, acts, N / 128, w2s, block_start, expert_counts, E, N, K,
                                      (int)ceil_div(K, 256), rows_cap, y_slots, nullptr, sorted_pairs, status, st);
  }
  if (!make_fp8_map(&mbm, w2q, 3, b_dims, b_str, 128)) return cudaErrorInvalidValue;
  return launch_f8_t<F8_GEMM2, 128>(ma, mbm, acts, N / 128, w2s, block_start, expert_counts, E, N, K,
                                    (int)ceil_div(K, 128), rows_cap, y_slots, nullptr, sorted_pairs, status, st);
}

}  // namespace moe

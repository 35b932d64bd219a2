// FP8 w8a8 expert GEMMs for decode-sized batches: weights as the MMA's M operand.
//
// Same math as moe_gemm_fp8.cu (DeepSeek-V3 recipe, fused_moe/v0/fused_moe.py:160-163 on
// dequantised operands):  D[n, t] = sum over 128-wide K blocks kb of
//   sw[n / 128, kb] * sa[t, kb] * P_kb[n, t],   P_kb = e4m3 x e4m3 products summed in fp32.
// With a few tokens per expert the token-major tiles are almost all padding and, worse,
// their 128 x 256 fp32 partial per K block leaves room for only two of them in TMEM, so
// the MMA can run one K block ahead of the CUDA-core promotion and the weight stream
// stalls on it. Here a tile is 128 weight rows x (up to) 32 tokens of one expert:
//   * a K block's partial is 128 x 32 (GEMM1: gate and up, 64 columns), so 8 partial slots
//     fit in TMEM and the MMA runs up to 7 K blocks ahead of the promotion;
//   * the promotion is 32 (GEMM1: 64) FMAs per thread and K block;
//   * every stage is 128-byte K slices of the weight rows (16 KB, twice for GEMM1's gate
//     and up rows), of the 32 token rows (4 KB) and their 32 row scales (128 B).
// Tiles: expert e, weight-row block cb (GEMM1: 128 intermediate channels, gate and up;
// GEMM2: 128 hidden columns), token chunk c (rows 32c .. 32c + 31 of the expert's
// segment). Tile order: expert, row block, chunk fastest.
//
//   warp 0      TMA producer (weights, token rows, row scales per stage)
//   warp 1      MMA issuer: tcgen05.mma.kind::f8f6f4, M = 128, N = 32, K = 32, 4 per
//               K block (GEMM1: 4 for gate + 4 for up) into partial slot kb % 8
//   warp 2      TMEM allocator; warp 3 builds the tile table
//   warps 4-7   promotion + tile epilogue, thread = weight row (TMEM lane), 32 token
//               totals per thread. GEMM1: act = SiLU(gate) * up, quantised per token per
//               128 channels (the tile's 128 channels; amax over the 4 warps) into e4m3 act
//               rows + scales ([channel blocks][rows] table). GEMM2: bf16 pair-slot rows.
// Outputs use the layouts of moe_gemm_fp8.cu, for the rows the align stage filled (the
// padding rows of a chunk are computed and dropped).
// Every mbarrier wait is bounded (common.cuh).
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>
#include <cuda_fp8.h>

namespace moe {
namespace {

enum { SW_GEMM1 = 0, SW_GEMM2 = 1 };

constexpr int kSwThreads = 256;
constexpr int kSwTok = 32;     // tokens per tile (MMA N)
constexpr int kSwBK = 128;     // K bytes per stage: one scale block
constexpr int kSwRows = 128;   // weight rows per tile (MMA M)
constexpr int kSwParts = 8;    // TMEM partial slots

__device__ __forceinline__ void umma_f8_sw(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::f8f6f4 instruction descriptor: A and B e4m3, D fp32, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_sw(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int MODE>
struct SwCfg {
  static constexpr int kATiles = MODE == SW_GEMM1 ? 2 : 1;  // gate + up, or w2
  static constexpr int kATile = kSwRows * kSwBK;             // 16 KB
  static constexpr int kBTile = kSwTok * kSwBK;              // 4 KB
  static constexpr int kScale = kSwTok * 4;                  // 128 B
  static constexpr int kTx = kATiles * kATile + kBTile + kScale;
  static constexpr int kStage = (kTx + 1023) / 1024 * 1024;  // tiles stay 1024-byte aligned
  static constexpr int kStages = MODE == SW_GEMM1 ? 5 : 8;
  static constexpr int kPartCols = kATiles * kSwTok;          // 64 / 32
  static constexpr uint32_t kTmemCols = MODE == SW_GEMM1 ? 512 : 256;
  static constexpr int kEpiOffset = kStages * kStage;
  // epilogue: GEMM1 [32 tokens][128 channels] e4m3 + amax [4 warps][32]; GEMM2 [32][128] bf16
  static constexpr int kEpiBytes = MODE == SW_GEMM1 ? kSwTok * 128 + 4 * kSwTok * 4 : kSwTok * 128 * 2;
  static constexpr int kBarOffset = kEpiOffset + kEpiBytes;
  static constexpr int kNumBars = 2 * kStages + 2 * kSwParts + 1;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kTableOffset = kMiscOffset + 16;
  static int bytes(int E) { return 1024 + kTableOffset + 3 * 4 * (E + 1); }
};

// tile -> expert e, row block rb, chunk c (chunk fastest); s_tp: prefix over experts of chunks
__device__ __forceinline__ void decode_sw_tile(const int* s_tp, int E, int NB, int tile, int& e, int& rb, int& c) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_tp[mid] * NB <= tile) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int nch = s_tp[lo + 1] - s_tp[lo];
  const int local = tile - s_tp[lo] * NB;
  rb = local / nch;
  c = local - rb * nch;
}

// MODE SW_GEMM1: map_a = w1 (K, N, 2E) box 128 rows; map_b = xq_sorted (K, rows); map_s = xs^T
// (rows, K/128) box 32; out = act_q [rows, N] e4m3, out_scale = act_s^T [N/128][rows_cap].
// MODE SW_GEMM2: map_a = w2 (N, K, E) box 128; map_b = act_q (N, rows); map_s = act_s^T; out =
// y slots [pairs, K] bf16 (row = sorted_pairs[r]).
// k_red: K bytes reduced (GEMM1 K, GEMM2 N); n_w: weight rows per expert half (GEMM1 N, GEMM2 K).
template <int MODE>
__global__ void __launch_bounds__(kSwThreads, 1)
moe_gemm_fp8_swap_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_s, const float* __restrict__ w_scale,
                         const int32_t* __restrict__ counts, const int32_t* __restrict__ block_start, int E,
                         int k_red, int n_w, int NB, void* __restrict__ out, float* __restrict__ out_scale,
                         int64_t rows_cap, const int32_t* __restrict__ sorted_pairs, bool pow2_act, int* status) {
  using C = SwCfg<MODE>;
  constexpr int S = C::kStages;
  constexpr uint32_t kIdesc = idesc_e4m3_sw(kSwRows, kSwTok);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + S;
  uint64_t* pfull = full + 2 * S;
  uint64_t* pempty = pfull + kSwParts;
  uint64_t* mma_done = pempty + kSwParts;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kMiscOffset);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::kMiscOffset + 4);
  int* s_bs = reinterpret_cast<int*>(smem + C::kTableOffset);  // [E + 1] m-block starts
  int* s_cnt = s_bs + (E + 1);                                 // [E] rows per expert
  int* s_tp = s_cnt + (E + 1);                                 // [E + 1] prefix of chunks

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i <= E; i += kSwThreads) {
    s_bs[i] = __ldg(block_start + i);
    if (i < E) s_cnt[i] = __ldg(counts + i);
  }
  if (threadIdx.x == 0) {
    // a stage is free once its MMAs completed and every epilogue warp read its row scales
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1 + 4); }
    for (int p = 0; p < kSwParts; ++p) { mbar_init(&pfull[p], 1); mbar_init(&pempty[p], 4); }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&map_a); tma_prefetch_desc(&map_b); tma_prefetch_desc(&map_s); }
  if (warp == 2) { tmem_alloc(s_tmem, C::kTmemCols); tmem_relinquish(); }
  __syncthreads();  // s_bs, s_cnt
  if (warp == 3) {  // s_tp[e] = sum over e' < e of ceil(count / 32); one warp, E <= 1024
    const int per = (E + 31) / 32;
    const int b = lane * per;
    int local = 0;
    for (int i = 0; i < per; ++i)
      if (b + i < E) local += (s_cnt[b + i] + kSwTok - 1) / kSwTok;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - local;
    for (int i = 0; i < per; ++i) {
      if (b + i < E) {
        s_tp[b + i] = run;
        run += (s_cnt[b + i] + kSwTok - 1) / kSwTok;
      }
    }
    if (lane == 31) s_tp[E] = incl;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_tiles = s_tp[E] * NB;
  const int num_kb = k_red / kSwBK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        int e, rb, c;
        decode_sw_tile(s_tp, E, NB, tile, e, rb, c);
        const int row0 = s_bs[e] * kBlockM + c * kSwTok;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
          uint8_t* st = smem + stage * C::kStage;
          mbar_arrive_expect_tx(&full[stage], C::kTx);
          if constexpr (MODE == SW_GEMM1) {
            tma_load_3d(&map_a, &full[stage], st, kb * kSwBK, rb * kSwRows, 2 * e);                // gate rows
            tma_load_3d(&map_a, &full[stage], st + C::kATile, kb * kSwBK, rb * kSwRows, 2 * e + 1);  // up rows
          } else {
            tma_load_3d(&map_a, &full[stage], st, kb * kSwBK, rb * kSwRows, e);
          }
          tma_load_2d(&map_b, &full[stage], st + C::kATiles * C::kATile, kb * kSwBK, row0);
          tma_load_2d(&map_s, &full[stage], st + C::kATiles * C::kATile + C::kBTile, row0, kb);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        for (int s = 0; s < S; ++s)
          if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0, part = 0;
      uint32_t phase = 0, pphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&pempty[part], pphase ^ 1, status, s_abort)) { ok = false; break; }
          if (!mbar_wait(&full[stage], phase, status, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* st = smem + stage * C::kStage;
          const uint64_t b_desc = smem_desc_sw128(st + C::kATiles * C::kATile);
          const uint32_t d = tmem_base + (uint32_t)(part * C::kPartCols);
#pragma unroll
          for (int a = 0; a < C::kATiles; ++a) {
            const uint64_t a_desc = smem_desc_sw128(st + a * C::kATile);
#pragma unroll
            for (int k = 0; k < kSwBK / 32; ++k)  // 32 e4m3 per MMA: +32 B = +2 in the start-address field
              umma_f8_sw(d + (uint32_t)(a * kSwTok), a_desc + 2 * k, b_desc + 2 * k, kIdesc, k != 0);
          }
          umma_commit(&empty[stage]);
          umma_commit(&pfull[part]);
          if (++stage == S) { stage = 0; phase ^= 1; }
          if (++part == kSwParts) { part = 0; pphase ^= 1; }
        }
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, nullptr);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ promotion + epilogue
    const int ew = warp - 4;
    const int wrow = ew * 32 + lane;  // this thread's weight row in the tile (TMEM lane)
    const int kbs = k_red / kSwBK;    // K blocks of the reduction (scale columns)
    uint8_t* epi = smem + C::kEpiOffset;
    int stage = 0, part = 0;
    uint32_t sphase = 0, pphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      int e, rb, c;
      decode_sw_tile(s_tp, E, NB, tile, e, rb, c);
      const int row0 = s_bs[e] * kBlockM + c * kSwTok;
      const int nvalid = min(kSwTok, s_cnt[e] - c * kSwTok);
      // weight block scales of this tile's row block(s), one per K block
      const float* sw0;
      const float* sw1;
      if constexpr (MODE == SW_GEMM1) {
        const int nrb = 2 * (n_w / 128);  // w1 row blocks per expert: gate blocks, then up blocks
        sw0 = w_scale + ((int64_t)e * nrb + rb) * kbs;
        sw1 = w_scale + ((int64_t)e * nrb + n_w / 128 + rb) * kbs;
      } else {
        sw0 = w_scale + ((int64_t)e * (n_w / 128) + rb) * kbs;
        sw1 = sw0;
      }
      float t0[kSwTok], t1[kSwTok];
#pragma unroll
      for (int j = 0; j < kSwTok; ++j) { t0[j] = 0.f; t1[j] = 0.f; }
      for (int kb = 0; kb < num_kb && ok; ++kb) {
        // the 32 token scales of this K block, then this warp's hold on the stage ends
        if (!mbar_wait(&full[stage], sphase, status, s_abort)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        float sa[kSwTok];
        const float4* ssc = reinterpret_cast<const float4*>(smem + stage * C::kStage + C::kATiles * C::kATile + C::kBTile);
#pragma unroll
        for (int q = 0; q < kSwTok / 4; ++q) {
          const float4 v = ssc[q];
          sa[4 * q] = v.x; sa[4 * q + 1] = v.y; sa[4 * q + 2] = v.z; sa[4 * q + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == S) { stage = 0; sphase ^= 1; }
        const float w0 = __ldg(sw0 + kb), w1v = __ldg(sw1 + kb);
        if (!mbar_wait(&pfull[part], pphase, status, s_abort)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(part * C::kPartCols);
        uint32_t v0[32];
        tmem_ld32(taddr, v0);
        if constexpr (MODE == SW_GEMM1) {
          uint32_t v1[32];
          tmem_ld32(taddr + kSwTok, v1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[part]);
#pragma unroll
          for (int j = 0; j < kSwTok; ++j) {
            t0[j] = fmaf(__uint_as_float(v0[j]), w0 * sa[j], t0[j]);
            t1[j] = fmaf(__uint_as_float(v1[j]), w1v * sa[j], t1[j]);
          }
        } else {
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[part]);
#pragma unroll
          for (int j = 0; j < kSwTok; ++j) t0[j] = fmaf(__uint_as_float(v0[j]), w0 * sa[j], t0[j]);
        }
        if (++part == kSwParts) { part = 0; pphase ^= 1; }
      }
      // every epilogue warp gets here (its waits are bounded) and they stop together
      ok = named_bar_and(1, 128, ok);
      if (!ok) break;
      if constexpr (MODE == SW_GEMM1) {
        // act = SiLU(gate) * up for channel rb * 128 + wrow and the chunk's 32 tokens;
        // per-token amax over the 128 channels: 32 warp reductions, then the 4 warps in smem
        float* s_amax = reinterpret_cast<float*>(epi + kSwTok * 128);  // [4][32]
        float my_amax = 0.f;  // lane j ends up with token j's amax over this warp
#pragma unroll
        for (int j = 0; j < kSwTok; ++j) {
          const float g = t0[j];
          t0[j] = g / (1.0f + __expf(-g)) * t1[j];
          float m = fabsf(t0[j]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == j) my_amax = m;
        }
        s_amax[ew * kSwTok + lane] = my_amax;
        named_bar_sync(1, 128);
        float sc[kSwTok];
#pragma unroll
        for (int j = 0; j < kSwTok; ++j) {
          const float a = fmaxf(fmaxf(s_amax[j], s_amax[kSwTok + j]), fmaxf(s_amax[2 * kSwTok + j], s_amax[3 * kSwTok + j]));
          sc[j] = fp8_block_scale(a, pow2_act);
        }
        // codes staged as [token][channel] bytes
#pragma unroll
        for (int j = 0; j < kSwTok; ++j) {
          const uint32_t q2 = __nv_cvt_float2_to_fp8x2(make_float2(t0[j] / sc[j], 0.f), __NV_SATFINITE, __NV_E4M3);
          epi[j * 128 + wrow] = (uint8_t)(q2 & 0xffu);
        }
        if (ew == 0 && lane < nvalid) {  // token `lane`'s scale, read from the amax table (no dynamic index)
          const float a = fmaxf(fmaxf(s_amax[lane], s_amax[kSwTok + lane]),
                                fmaxf(s_amax[2 * kSwTok + lane], s_amax[3 * kSwTok + lane]));
          out_scale[(int64_t)rb * rows_cap + row0 + lane] = fp8_block_scale(a, pow2_act);
        }
        named_bar_sync(1, 128);
        // 32 token rows x 128 bytes -> act rows (row0 + j, channels rb * 128 ..)
        uint8_t* act = static_cast<uint8_t*>(out);
        const int et = threadIdx.x - 128;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int ch = et + 128 * i;  // 16-byte chunk id: token ch / 8, chunk ch % 8
          const int j = ch >> 3, q = ch & 7;
          if (j < nvalid)
            *reinterpret_cast<uint4*>(act + (int64_t)(row0 + j) * n_w + rb * 128 + q * 16) =
                *reinterpret_cast<const uint4*>(epi + j * 128 + q * 16);
        }
        named_bar_sync(1, 128);
      } else {
        // bf16 output column rb * 128 + wrow for the chunk's 32 tokens, staged [token][column]
        __nv_bfloat16* s_y = reinterpret_cast<__nv_bfloat16*>(epi);
#pragma unroll
        for (int j = 0; j < kSwTok; ++j) s_y[j * 128 + wrow] = __float2bfloat16_rn(t0[j]);
        named_bar_sync(1, 128);
        __nv_bfloat16* y = static_cast<__nv_bfloat16*>(out);
        const int et = threadIdx.x - 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ch = et + 128 * i;  // token ch / 16, 16-byte chunk ch % 16
          const int j = ch >> 4, q = ch & 15;
          if (j < nvalid) {
            const int pair = __ldg(sorted_pairs + row0 + j);
            if (pair >= 0)
              *reinterpret_cast<uint4*>(y + (int64_t)pair * n_w + rb * 128 + q * 8) =
                  *reinterpret_cast<const uint4*>(s_y + j * 128 + q * 8);
          }
        }
        named_bar_sync(1, 128);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int MODE>
cudaError_t launch_sw(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& ms, const float* w_scale,
                      const int32_t* counts, const int32_t* block_start, int E, int k_red, int n_w, int NB,
                      int64_t rows_cap, int64_t num_pairs, void* out, float* out_scale, const int32_t* sorted_pairs,
                      bool pow2_act, int* status, int max_ctas, cudaStream_t st) {
  using C = SwCfg<MODE>;
  auto kern = moe_gemm_fp8_swap_kernel<MODE>;
  const int smem = C::bytes(E);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t err = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
  if (err != cudaSuccess) return err;
  const int64_t tiles_cap = (ceil_div(num_pairs, kSwTok) + E) * (int64_t)NB;  // chunks <= pairs / 32 + E
  const int ctas = (max_ctas > 0 && max_ctas < num_sms()) ? max_ctas : num_sms();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas, tiles_cap));
  kern<<<grid, kSwThreads, smem, st>>>(ma, mb, ms, w_scale, counts, block_start, E, k_red, n_w, NB, out, out_scale,
                                       rows_cap, sorted_pairs, pow2_act, status);
  return cudaGetLastError();
}

// [K blocks][rows_cap] fp32 scale table with a 32-row box.
bool make_scale_map32(CUtensorMap* m, const float* base, int64_t rows_cap, int kblocks) {
  const uint64_t dims[2] = {(uint64_t)rows_cap, (uint64_t)kblocks};
  const uint64_t str[1] = {(uint64_t)rows_cap * 4};
  return make_f32_rows_map(m, base, dims, str, kSwTok);
}

}  // namespace

bool fp8_use_swap(int64_t num_pairs, int E) { return num_pairs <= kFp8SwapMaxRowsPerExpert * (int64_t)E; }

cudaError_t launch_fp8_swap_gemm1(const void* xq_sorted, const float* xs_sorted_t, int64_t rows_cap,
                                  int64_t num_pairs, const void* w1q, const float* w1s, int E, int K, int N,
                                  const int32_t* counts, const int32_t* block_start, void* actq, float* acts_t,
                                  bool pow2_act, int* status, int max_ctas, cudaStream_t st) {
  CUtensorMap ma, mbm, ms;
  const uint64_t a_dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)2 * E};
  const uint64_t a_str[2] = {(uint64_t)K, (uint64_t)N * K};
  const uint64_t b_dims[2] = {(uint64_t)K, (uint64_t)rows_cap};
  const uint64_t b_str[1] = {(uint64_t)K};
  if (!make_fp8_map(&ma, w1q, 3, a_dims, a_str, kSwRows)) return cudaErrorInvalidValue;
  if (!make_fp8_map(&mbm, xq_sorted, 2, b_dims, b_str, kSwTok)) return cudaErrorInvalidValue;
  if (!make_scale_map32(&ms, xs_sorted_t, rows_cap, K / 128)) return cudaErrorInvalidValue;
  return launch_sw<SW_GEMM1>(ma, mbm, ms, w1s, counts, block_start, E, K, N, N / 128, rows_cap, num_pairs, actq,
                             acts_t, nullptr, pow2_act, status, max_ctas, st);
}

cudaError_t launch_fp8_swap_gemm2(const void* actq, const float* acts_t, int64_t rows_cap, int64_t num_pairs,
                                  const void* w2q, const float* w2s, int E, int K, int N, const int32_t* counts,
                                  const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots, int* status,
                                  int max_ctas, cudaStream_t st) {
  CUtensorMap ma, mbm, ms;
  const uint64_t a_dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)E};
  const uint64_t a_str[2] = {(uint64_t)N, (uint64_t)K * N};
  const uint64_t b_dims[2] = {(uint64_t)N, (uint64_t)rows_cap};
  const uint64_t b_str[1] = {(uint64_t)N};
  if (!make_fp8_map(&ma, w2q, 3, a_dims, a_str, kSwRows)) return cudaErrorInvalidValue;
  if (!make_fp8_map(&mbm, actq, 2, b_dims, b_str, kSwTok)) return cudaErrorInvalidValue;
  if (!make_scale_map32(&ms, acts_t, rows_cap, N / 128)) return cudaErrorInvalidValue;
  return launch_sw<SW_GEMM2>(ma, mbm, ms, w2s, counts, block_start, E, N, K, K / 128, rows_cap, num_pairs, y_slots,
                             nullptr, sorted_pairs, false, status, max_ctas, st);
}

}  // namespace moe

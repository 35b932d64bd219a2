// Grouped expert GEMMs for the FP8 w8a8 configuration (DeepSeek-V3 recipe:
// e4m3 weights with an fp32 scale per 128 x 128 block, e4m3 activations with an
// fp32 scale per token per 128 channels). The math is the expert path of
// fused_moe/v0/fused_moe.py:160-163 on dequantised operands:
//   D[m, n] = sum over 128-wide K blocks kb of  sa[m, kb] * sw[n / 128, kb] * P_kb[m, n],
//   P_kb[m, n] = sum over k in kb of qa[m, k] * qb[n, k]      (e4m3 x e4m3 -> fp32)
//
// tcgen05's block-scaled MMA kinds take power-of-two scales per 32 elements and
// cannot carry an fp32 scale per 128 x 128 block, so every K block is one chain
// of tcgen05.mma.kind::f8f6f4 (e4m3 operands straight from shared memory) into
// a TMEM partial accumulator, and the epilogue warps promote it: they read the
// partial and add it, times sa * sw, into fp32 totals held in registers. Two
// partial buffers let the MMAs of block kb + 1 run while block kb is promoted.
//
//   warp 0      TMA producer: one 128-wide K block per stage, A = 128 rows x 128 B,
//               B = 256 rows x 128 B, 128-byte swizzle, plus the K block's 128 row
//               scales (one 512-byte row of a [K blocks][rows] table). GEMM1 stacks
//               the B rows as [gate 0..63 | up 0..63 | gate 64..127 | up 64..127] of
//               the tile's 128 intermediate channels, so each epilogue warpgroup owns
//               the gate and up columns of the same 64 channels.
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (M=128, N=256, K=32) per
//               stage into partial buffer kb & 1.
//   warp 2      TMEM allocator (2 partial buffers x 256 fp32 columns); warp 3 idle.
//   warps 4-11  promotion + tile epilogue; warp w reads TMEM lanes 32 * (w % 4)
//               (one row per thread) and columns 128 * h, h = (w - 4) / 4: 128 fp32
//               totals per thread, updated with packed fp32 FMAs. A stage is free
//               once its MMAs completed and every epilogue warp read its row scales.
//               Warpgroup 0 (warps 0-3) gives registers back (setmaxnreg 40) so the
//               two epilogue warpgroups can hold 232 each.
//               GEMM1: act = SiLU(gate) * up in fp32, quantised per row per 128
//               channels (scale = amax / 448, the two warpgroups' halves of the
//               amax meet in shared memory) -> e4m3 act rows + scales ([channel
//               blocks][rows] table), the A operand of GEMM2. GEMM2: bf16 rows of
//               the pair slots. Stores are staged per warp in shared memory and
//               leave as 64-byte row segments.
//
// Where the time goes (measured on B200, DeepSeek-V3 shapes): with the promotion
// removed the two GEMMs run near the e4m3 tensor rate; the promotion's fp32 work
// (128 x 256 FMAs per 128-wide K block, on the CUDA cores, between a partial's
// tcgen05.ld and its buffer's release) is as long as the MMAs it has to overlap,
// and with two buffers the MMA waits for it part of the time.
//
// Block-scaled variant (MX = true), for weights whose every scale is a power of
// two (UE8M0, the block-scale format of tcgen05's kind::mxf8f6f4; DeepSeek's
// format on Blackwell), with the activations quantised the same way: the tensor
// cores apply the scales, one MMA chain accumulates the whole K into a single
// 256-column TMEM accumulator, and there is no promotion.
//   warp 0      all 32 lanes write the stage's B scale-factor atoms (the UE8M0
//               codes of the tile's weight blocks) into shared memory; lane 0
//               loads A, B and the A scale-factor atom (512 B) by TMA.
//   warp 1      per stage: tcgen05.cp of the A atom (TMEM columns 256 + 16 s ..
//               + 3 for stage s) and the two B atoms (the next 8 columns), then
//               4 x tcgen05.mma.kind::mxf8f6f4.
//               block_scale (M=128, N=256, K=32), K chunk k reading scale byte k.
//   warps 4-11  wait for the tile's accumulator, read it (128 columns per thread),
//               hand it back and run the same tile epilogue (act scales are
//               powers of two, written as scale-factor atoms for GEMM2).
// A scale-factor atom holds the 128 rows x 4 K chunks of one m-block and K block:
// row r's code at byte (r % 32) * 16 + (r / 32) * 4 + chunk; tcgen05.cp's
// 32x128b.warpx4 shape copies it to TMEM lanes r % 32 of every 32-lane quarter,
// column r / 32, byte = chunk, where the MMA reads it.
// Rows come from the align stage (pairs grouped by expert, 128-row m-blocks).
// All mbarrier waits are bounded (common.cuh); the one named barrier of the
// epilogue is an AND-reduction, so a warp that gave up makes all of them stop.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>
#include <cuda_fp8.h>

namespace moe {
namespace {

enum { F8_GEMM1 = 0, F8_GEMM2 = 1 };

constexpr int kF8Threads = 384;
constexpr int kF8BK = 128;                   // K elements (= bytes) per stage: one scale block
constexpr int kF8BN = 256;                   // MMA N
constexpr int kF8ATile = kBlockM * kF8BK;    // 16 KB
constexpr int kF8BTile = kF8BN * kF8BK;      // 32 KB
constexpr int kF8Stage = kF8ATile + kF8BTile;
constexpr int kF8EpiWarps = 8;
constexpr int kF8StageRowBytes = 64;         // epilogue staging: 32 rows x 64 B per warp
constexpr int kF8EpiWarpBytes = 32 * kF8StageRowBytes;

template <int STAGES, bool MX = false>
struct F8Smem {
  static constexpr int kEpiOffset = STAGES * kF8Stage;
  static constexpr int kAmaxOffset = kEpiOffset + kF8EpiWarps * kF8EpiWarpBytes;  // [2 tiles][2 halves][128] fp32
  static constexpr int kAScaleOffset = kAmaxOffset + 2 * 2 * 128 * 4;             // [STAGES][128] fp32 row scales
                                                                                  // (MX: A scale-factor atoms)
  static constexpr int kSfbOffset = kAScaleOffset + STAGES * 128 * 4;             // MX: [STAGES][2 atoms][512 B]
  static constexpr int kBarOffset = kSfbOffset + (MX ? STAGES * 1024 : 0);
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kTableOffset = kMiscOffset + 16;
  static int bytes(int E) { return 1024 + kTableOffset + 4 * (E + 1); }
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

// D[tmem] (+)= A[smem] * B[smem]^T with e4m3 operands and fp32 accumulation.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor of kind::f8f6f4: A and B e4m3 (format code 0), D fp32,
// both K-major; the N and M fields sit where they do for kind::f16.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// kind::mxf8f6f4.block_scale: D[tmem] (+)= (A * 2^sfa) * (B * 2^sfb)^T per 32-wide K chunk,
// e4m3 operands, UE8M0 scale factors read from TMEM (sfa, sfb carry the byte of the
// chunk in their top two bits, as the descriptor's scale-factor ids do).
__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// Instruction descriptor of kind::mxf8f6f4.block_scale: A and B e4m3, UE8M0 scale
// factors, both K-major, scale-factor byte sf of the A and B scale words.
__host__ __device__ constexpr uint32_t idesc_mx_e4m3(int M, int N, int sf) {
  return ((uint32_t)sf << 4)               // B scale-factor id
         | ((uint32_t)(N >> 3) << 17)      // N >> 3
         | (1u << 23)                      // scale format: UE8M0
         | ((uint32_t)(M >> 4) << 24)      // M >> 4
         | ((uint32_t)sf << 29);           // A scale-factor id
}

// Copies a 32-row x 16-byte shared-memory matrix into TMEM columns [taddr, taddr + 4)
// of lanes 0-31, replicated into each of the four 32-lane quarters.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Shared-memory descriptor of a scale-factor atom for tcgen05.cp: no swizzle, rows of
// 16 bytes, 8-row core matrices 128 B apart.
__device__ __forceinline__ uint64_t smem_desc_sf(const void* p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = (addr >> 4) & 0x3FFFull;  // bits [0,14): start address >> 4
  d |= (uint64_t)(128 >> 4) << 32;       // bits [32,46): stride byte offset = 128 B
  d |= 1ull << 46;                       // bits [46,48): descriptor version 1 (sm_100); layout 0: no swizzle
  return d;
}

// Byte offset of 16-byte chunk c (0..3) of staged row r (32 rows x 64 B): the
// chunk index is XORed with (r >> 1) & 3 so that 8 consecutive rows written at
// the same chunk fall in 8 distinct 16-byte bank groups.
__device__ __forceinline__ int stage_off(int r, int c) { return r * kF8StageRowBytes + ((c ^ ((r >> 1) & 3)) << 4); }

// tcgen05.wait::ld that also names the destination registers of the load it
// waits for, so the compiler cannot move their uses above the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Ties the registers of a second tcgen05.ld to a point after the preceding wait (both asm
// statements are volatile, so they keep their order): uses of r cannot move above it.
__device__ __forceinline__ void reg_order32(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// tot[p0 + i] += (v[2i], v[2i + 1]) * f for i < 16: 32 partial columns into 16 fp32 pairs.
__device__ __forceinline__ void promote32(float2 (&tot)[64], int p0, const uint32_t (&v)[32], float2 f) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    tot[p0 + i] = __ffma2_rn(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), f, tot[p0 + i]);
}

constexpr int kF8RegsLaunch = 168;  // 65536 / 384 rounded down to a multiple of 8
constexpr int kF8RegsLow = 40;
constexpr int kF8RegsHigh = 232;
static_assert(128 * kF8RegsLow + 256 * kF8RegsHigh <= kF8Threads * kF8RegsLaunch, "register split exceeds the launch");
static_assert(kF8BN + 4 * 16 <= 512, "accumulator and four scale-factor slots fit the TMEM allocation");

template <int R> __device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(R));
}
template <int R> __device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(R));
}

template <int MODE, int STAGES, bool MX>
__global__ void __launch_bounds__(kF8Threads, 1)
moe_gemm_fp8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_sa, const float* __restrict__ b_scale,
                    const int32_t* __restrict__ block_start, int E, int k_red, int n_out, int NB,
                    void* __restrict__ out, float* __restrict__ out_scale, int64_t out_scale_stride,
                    const int32_t* __restrict__ sorted_pairs, int* status) {
  using L = F8Smem<STAGES, MX>;
  constexpr int kBatch = 1;  // K blocks whose row scales the epilogue reads at once (measured: 1 is fastest)
  constexpr uint32_t kTmemCols = 2 * kF8BN;
  constexpr uint32_t kIdesc = idesc_e4m3(kBlockM, kF8BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = full + 2 * STAGES;  // partial accumulator b holds a finished K block (MX: [0] tile done)
  uint64_t* pempty = pfull + 2;         // partial accumulator b has been promoted (MX: [0] tile read out)
  uint64_t* mma_done = pfull + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);
  int* s_bs = reinterpret_cast<int*>(smem + L::kTableOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i <= E; i += kF8Threads) s_bs[i] = __ldg(block_start + i);
  if (threadIdx.x == 0) {
    // a stage is free once its MMAs finished (commit) and every epilogue warp read its row
    // scales (MX: once its MMAs and scale-factor copies finished)
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], MX ? 1 : 1 + kF8EpiWarps); }
    for (int b = 0; b < 2; ++b) { mbar_init(&pfull[b], 1); mbar_init(&pempty[b], kF8EpiWarps); }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&map_a); tma_prefetch_desc(&map_b); tma_prefetch_desc(&map_sa); }
  if (warp == 2) { tmem_alloc(s_tmem, kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_tiles = s_bs[E] * NB;
  const int num_kb = (k_red + kF8BK - 1) / kF8BK;
  // Register split: 128 x 40 + 256 x 232 = 384 x 168, the launch's allocation (the host
  // refuses to launch unless the kernel was compiled to exactly 168 registers per thread).
  if (warp < 4) {
    setmaxnreg_dec<kF8RegsLow>();
  if (warp == 0 && MX) {
    // ------------------------------------------------ TMA producer + B scale-factor atoms (MX)
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool ok = true;
    const int kb128 = (k_red + 127) / 128;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      int e, nb, mb;
      decode_tile_f8(s_bs, E, NB, tile, e, nb, mb);
      // the weight blocks of the tile's B rows: GEMM1 rows [gate | up | gate | up] x 64 come
      // from one gate and one up block; GEMM2's 256 rows from two consecutive row blocks
      const float* sw_lo;
      const float* sw_hi;
      if constexpr (MODE == F8_GEMM1) {
        const int nrb = 2 * (n_out / 128);
        sw_lo = b_scale + ((int64_t)e * nrb + nb) * kb128;
        sw_hi = b_scale + ((int64_t)e * nrb + n_out / 128 + nb) * kb128;
      } else {
        const int nblk = (n_out + 127) / 128;
        sw_lo = b_scale + ((int64_t)e * nblk + 2 * nb) * kb128;
        sw_hi = b_scale + ((int64_t)e * nblk + min(2 * nb + 1, nblk - 1)) * kb128;
      }
      const float wl_r0 = lane < kb128 ? __ldg(sw_lo + lane) : 1.f;
      const float wl_r1 = lane + 32 < kb128 ? __ldg(sw_lo + lane + 32) : 1.f;
      const float wh_r0 = lane < kb128 ? __ldg(sw_hi + lane) : 1.f;
      const float wh_r1 = lane + 32 < kb128 ? __ldg(sw_hi + lane + 32) : 1.f;
      for (int kb = 0; kb < num_kb; ++kb) {
        const bool got = mbar_wait(&empty[stage], phase ^ 1, status, s_abort);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        float wl, wh;
        if (kb < 64) {
          wl = __shfl_sync(0xffffffffu, kb < 32 ? wl_r0 : wl_r1, kb & 31);
          wh = __shfl_sync(0xffffffffu, kb < 32 ? wh_r0 : wh_r1, kb & 31);
        } else {
          wl = __ldg(sw_lo + kb);
          wh = __ldg(sw_hi + kb);
        }
        const uint32_t cl = ue8m0x4(wl), ch = ue8m0x4(wh);
        // atom words: column r / 32 of 16-byte row r % 32; GEMM1 rows 0-63 gate, 64-127 up
        uint4* sfb = reinterpret_cast<uint4*>(smem + L::kSfbOffset + stage * 1024);
        if constexpr (MODE == F8_GEMM1) {
          sfb[lane] = make_uint4(cl, cl, ch, ch);
          sfb[32 + lane] = make_uint4(cl, cl, ch, ch);
        } else {
          sfb[lane] = make_uint4(cl, cl, cl, cl);
          sfb[32 + lane] = make_uint4(ch, ch, ch, ch);
        }
        fence_proxy_async_smem();  // generic writes -> the async proxy of tcgen05.cp
        __syncwarp();
        if (lane == 0) {
          uint8_t* a_dst = smem + stage * kF8Stage;
          uint8_t* b_dst = a_dst + kF8ATile;
          mbar_arrive_expect_tx(&full[stage], kF8Stage + kBlockM * 4);
          tma_load_2d(&map_a, &full[stage], a_dst, kb * kF8BK, mb * kBlockM);
          tma_load_2d(&map_sa, &full[stage], smem + L::kAScaleOffset + stage * kBlockM * 4, mb * kBlockM, kb);
          if constexpr (MODE == F8_GEMM1) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              tma_load_3d(&map_b, &full[stage], b_dst + q * 64 * kF8BK, kb * kF8BK, nb * 128 + (q >> 1) * 64,
                          2 * e + (q & 1));
          } else {
            tma_load_3d(&map_b, &full[stage], b_dst, kb * kF8BK, nb * kF8BN, e);
          }
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && lane == 0) {  // let the copies in flight land before the CTA exits
      for (int s = 0; s < STAGES; ++s)
        if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, nullptr);
    }
  } else if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        int e, nb, mb;
        decode_tile_f8(s_bs, E, NB, tile, e, nb, mb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, s_abort)) { ok = false; break; }
          uint8_t* a_dst = smem + stage * kF8Stage;
          uint8_t* b_dst = a_dst + kF8ATile;
          mbar_arrive_expect_tx(&full[stage], kF8Stage + kBlockM * 4);
          tma_load_2d(&map_a, &full[stage], a_dst, kb * kF8BK, mb * kBlockM);
          // the 128 row scales of this K block: one 512-byte row of the [K blocks][rows] table
          tma_load_2d(&map_sa, &full[stage], smem + L::kAScaleOffset + stage * kBlockM * 4, mb * kBlockM, kb);
          if constexpr (MODE == F8_GEMM1) {
#pragma unroll
            for (int q = 0; q < 4; ++q)  // gate lo, up lo, gate hi, up hi: 64 rows x 128 B each
              tma_load_3d(&map_b, &full[stage], b_dst + q * 64 * kF8BK, kb * kF8BK, nb * 128 + (q >> 1) * 64,
                          2 * e + (q & 1));
          } else {
            tma_load_3d(&map_b, &full[stage], b_dst, kb * kF8BK, nb * kF8BN, e);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        for (int s = 0; s < STAGES; ++s)
          if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, nullptr);
      }
    }
  } else if (warp == 1 && MX) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer (MX): whole K into one accumulator
      int stage = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      // one 16-column scale-factor slot per stage (A: 4 columns, B: 8), so a stage's copies
      // never overwrite the factors the previous stage's MMAs are still reading
      const uint32_t sf_base = tmem_base + (uint32_t)kF8BN;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&pempty[0], aphase ^ 1, status, s_abort)) break;  // previous tile read out
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* a_src = smem + stage * kF8Stage;
          const uint64_t a_desc = smem_desc_sw128(a_src);
          const uint64_t b_desc = smem_desc_sw128(a_src + kF8ATile);
          const uint8_t* sfb = smem + L::kSfbOffset + stage * 1024;
          // issued by this thread ahead of the MMAs, which then read them in order
          const uint32_t sfa_t = sf_base + (uint32_t)(stage * 16), sfb_t = sfa_t + 4;
          tmem_cp_sf(sfa_t, smem_desc_sf(smem + L::kAScaleOffset + stage * kBlockM * 4));
          tmem_cp_sf(sfb_t, smem_desc_sf(sfb));
          tmem_cp_sf(sfb_t + 4, smem_desc_sf(sfb + 512));
#pragma unroll
          for (int k = 0; k < kF8BK / 32; ++k)
            umma_mx(tmem_base, a_desc + 2 * k, b_desc + 2 * k, idesc_mx_e4m3(kBlockM, kF8BN, k),
                    sfa_t + ((uint32_t)k << 30), sfb_t + ((uint32_t)k << 30), (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&pfull[0]);
        aphase ^= 1;
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0, pb = 0;
      uint32_t phase = 0, pphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&pempty[pb], pphase ^ 1, status, s_abort)) { ok = false; break; }
          if (!mbar_wait(&full[stage], phase, status, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* a_src = smem + stage * kF8Stage;
          const uint64_t a_desc = smem_desc_sw128(a_src);
          const uint64_t b_desc = smem_desc_sw128(a_src + kF8ATile);
          const uint32_t d_tmem = tmem_base + (uint32_t)(pb * kF8BN);
#pragma unroll
          for (int k = 0; k < kF8BK / 32; ++k)  // 32 e4m3 per MMA: +32 B = +2 in the start-address field
            umma_f8(d_tmem, a_desc + 2 * k, b_desc + 2 * k, kIdesc, k != 0);
          umma_commit(&empty[stage]);
          umma_commit(&pfull[pb]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
          if (++pb == 2) { pb = 0; pphase ^= 1; }
        }
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, nullptr);
    }
  }
  } else {
    setmaxnreg_inc<kF8RegsHigh>();
    // ------------------------------------------------ promotion + epilogue (warps 4..11)
    const int ew = warp - 4;
    const int quad = warp & 3;
    const int h = ew >> 2;
    const int row = quad * 32 + lane;
    uint8_t* stage_buf = smem + L::kEpiOffset + ew * kF8EpiWarpBytes;
    float* s_amax = reinterpret_cast<float*>(smem + L::kAmaxOffset);
    const int kb128 = (k_red + 127) / 128;
    const int rd_r = lane >> 2, rd_c = lane & 3;  // staged-read mapping: 8 rows x 4 chunks per instruction
    int pb = 0, tpar = 0, stage = 0;
    uint32_t pphase = 0, sphase = 0;
    const float* s_sa = reinterpret_cast<const float*>(smem + L::kAScaleOffset);
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, tpar ^= 1) {
      int e, nb, mb;
      decode_tile_f8(s_bs, E, NB, tile, e, nb, mb);
      const int64_t grow = (int64_t)mb * kBlockM + row;
      // totals as fp32 pairs: column 2j in .x, 2j + 1 in .y (packed FMA, two columns per instruction)
      float2 tot[64];
      bool cols_live = true;
      if constexpr (MODE == F8_GEMM2) cols_live = (2 * nb + h) * 128 < n_out;
      if constexpr (MX) {
        // the MMAs applied the scales: read the finished accumulator and hand it back
        bool got = mbar_wait(&pfull[0], pphase, status, s_abort);
        got = __all_sync(0xffffffffu, got);
        if (got) {
          tc_fence_after();
          const uint32_t t_addr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(h * 128);
          uint32_t va[32], vb[32];
          tmem_ld32(t_addr, va);
          tmem_ld32(t_addr + 32, vb);
          tmem_wait_ld_regs(va);
          reg_order32(vb);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            tot[i] = make_float2(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1]));
            tot[16 + i] = make_float2(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1]));
          }
          tmem_ld32(t_addr + 64, va);
          tmem_ld32(t_addr + 96, vb);
          tmem_wait_ld_regs(va);
          reg_order32(vb);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[0]);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            tot[32 + i] = make_float2(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1]));
            tot[48 + i] = make_float2(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1]));
          }
          pphase ^= 1;
        } else {
          ok = false;
#pragma unroll
          for (int j = 0; j < 64; ++j) tot[j] = make_float2(0.f, 0.f);
        }
      } else {
      // weight scales of the tile's K blocks: lane i holds blocks i and i + 32 (a shuffle
      // broadcasts block kb); blocks from 64 on are read per block
      const float* sw_lo;
      const float* sw_hi;
      if constexpr (MODE == F8_GEMM1) {
        const int nrb = 2 * (n_out / 128);  // w1 row blocks per expert: gate blocks, then up blocks
        sw_lo = b_scale + ((int64_t)e * nrb + nb) * kb128;
        sw_hi = b_scale + ((int64_t)e * nrb + n_out / 128 + nb) * kb128;
      } else {
        const int cblk = 2 * nb + h;
        sw_lo = b_scale + ((int64_t)e * ((n_out + 127) / 128) + (cols_live ? cblk : 0)) * kb128;
        sw_hi = sw_lo;
      }
      const float wl_r0 = lane < kb128 ? __ldg(sw_lo + lane) : 0.f;
      const float wl_r1 = lane + 32 < kb128 ? __ldg(sw_lo + lane + 32) : 0.f;
      const float wh_r0 = lane < kb128 ? __ldg(sw_hi + lane) : 0.f;
      const float wh_r1 = lane + 32 < kb128 ? __ldg(sw_hi + lane + 32) : 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j) tot[j] = make_float2(0.f, 0.f);
      float sa_q[kBatch];
      for (int kb = 0; kb < num_kb; ++kb) {
        if (kb % kBatch == 0) {
          // row scales of the next kBatch K blocks (they land with the operands, and the
          // producer is at least that far ahead), then release this warp's hold on those stages
          const int first = stage;
          const int nq = min(kBatch, num_kb - kb);
#pragma unroll
          for (int i = 0; i < kBatch; ++i) {
            if (i < nq) {
              if (!mbar_wait(&full[stage], sphase, status, s_abort)) ok = false;
              sa_q[i] = s_sa[stage * kBlockM + row];
              if (++stage == STAGES) { stage = 0; sphase ^= 1; }
            }
          }
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          __syncwarp();
          if (lane == 0)
            for (int i = 0, st = first; i < nq; ++i, st = (st + 1 == STAGES ? 0 : st + 1)) mbar_arrive(&empty[st]);
        }
        const float sa = sa_q[0];
#pragma unroll
        for (int i = 0; i + 1 < kBatch; ++i) sa_q[i] = sa_q[i + 1];
        float wl, wh;
        if (kb < 64) {
          wl = __shfl_sync(0xffffffffu, kb < 32 ? wl_r0 : wl_r1, kb & 31);
          wh = __shfl_sync(0xffffffffu, kb < 32 ? wh_r0 : wh_r1, kb & 31);
        } else {
          wl = __ldg(sw_lo + kb);
          wh = __ldg(sw_hi + kb);
        }
        const float2 f_lo = make_float2(sa * wl, sa * wl), f_hi = make_float2(sa * wh, sa * wh);
        if (!mbar_wait(&pfull[pb], pphase, status, s_abort)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const uint32_t t_addr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(pb * kF8BN + h * 128);
        // the 128 columns in two pairs of 32-column loads, each pair in flight together under
        // one wait (a wait per load left four load latencies in a row per K block)
        uint32_t va[32], vb[32];
        tmem_ld32(t_addr, va);
        tmem_ld32(t_addr + 32, vb);
        tmem_wait_ld_regs(va);
        reg_order32(vb);
        promote32(tot, 0, va, f_lo);
        promote32(tot, 16, vb, f_lo);
        tmem_ld32(t_addr + 64, va);
        tmem_ld32(t_addr + 96, vb);
        tmem_wait_ld_regs(va);
        reg_order32(vb);
        // the partial is in registers: hand the buffer back before the last FMAs
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pb]);
        promote32(tot, 32, va, f_hi);
        promote32(tot, 48, vb, f_hi);
        if (++pb == 2) { pb = 0; pphase ^= 1; }
      }
      }  // promotion
      if constexpr (MODE == F8_GEMM1) {
        // act for the 64 channels nb * 128 + 64 h + j, quantised per row per 128 channels
        // gate channel pairs in tot[0..31], the matching up pairs in tot[32..63]
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 g = tot[i], u = tot[32 + i];
          tot[i] = make_float2(g.x / (1.0f + __expf(-g.x)) * u.x, g.y / (1.0f + __expf(-g.y)) * u.y);
          amax = fmaxf(amax, fmaxf(fabsf(tot[i].x), fabsf(tot[i].y)));
        }
        s_amax[(tpar * 2 + h) * 128 + row] = amax;
        ok = named_bar_and(1, 32 * kF8EpiWarps, ok);
        if (!ok) break;
        amax = fmaxf(amax, s_amax[(tpar * 2 + (h ^ 1)) * 128 + row]);
        const float sc = fp8_block_scale(amax, MX);
        if (h == 0) {  // [channel blocks][rows]; MX: the rows of an m-block as a scale-factor atom
          if constexpr (MX)
            reinterpret_cast<uint32_t*>(out_scale)[(int64_t)nb * out_scale_stride + (int64_t)mb * kBlockM + lane * 4 +
                                                   quad] = ue8m0x4(sc);
          else
            out_scale[(int64_t)nb * out_scale_stride + grow] = sc;
        }
        uint32_t q[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(tot[2 * i].x / sc, tot[2 * i].y / sc),
                                                       __NV_SATFINITE, __NV_E4M3);
          const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(tot[2 * i + 1].x / sc, tot[2 * i + 1].y / sc),
                                                       __NV_SATFINITE, __NV_E4M3);
          q[i] = lo | (hi << 16);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(stage_buf + stage_off(lane, c)) =
              make_uint4(q[4 * c], q[4 * c + 1], q[4 * c + 2], q[4 * c + 3]);
        __syncwarp();
        uint8_t* act = static_cast<uint8_t*>(out);
        const int64_t row0 = (int64_t)mb * kBlockM + quad * 32;
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int r = it * 8 + rd_r;
          const uint4 val = *reinterpret_cast<const uint4*>(stage_buf + stage_off(r, rd_c));
          *reinterpret_cast<uint4*>(act + (row0 + r) * (int64_t)n_out + nb * 128 + h * 64 + rd_c * 16) = val;
        }
        __syncwarp();
      } else {
        if (!ok) break;
        __nv_bfloat16* y = static_cast<__nv_bfloat16*>(out);
        const int my_pair = __ldg(sorted_pairs + grow);
        const int col0 = nb * kF8BN + h * 128;
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // 4 groups of 32 output columns (64 B per row)
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            __nv_bfloat162 b = __floats2bfloat162_rn(tot[16 * g + i].x, tot[16 * g + i].y);
            packed[i] = *reinterpret_cast<uint32_t*>(&b);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stage_buf + stage_off(lane, c)) =
                make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int r = it * 8 + rd_r;
            const uint4 val = *reinterpret_cast<const uint4*>(stage_buf + stage_off(r, rd_c));
            const int pair = __shfl_sync(0xffffffffu, my_pair, r);
            if (pair >= 0 && cols_live)
              *reinterpret_cast<uint4*>(y + (int64_t)pair * n_out + col0 + 32 * g + rd_c * 8) = val;
          }
          __syncwarp();
        }
      }
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
gather_rows_kernel(const uint8_t* __restrict__ src, int64_t src_stride, int64_t row_bytes,
                   const int32_t* __restrict__ sorted_pairs, const int32_t* __restrict__ block_start, int E, int topk,
                   int64_t cap, uint8_t* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= cap || r >= (int64_t)__ldg(block_start + E) * kBlockM) return;
  const int pair = __ldg(sorted_pairs + r);
  if (pair < 0) return;
  const int64_t t = pair / topk;
  if ((row_bytes & 15) == 0 && (src_stride & 15) == 0) {
    const uint4* s = reinterpret_cast<const uint4*>(src + t * src_stride);
    uint4* d = reinterpret_cast<uint4*>(dst + r * row_bytes);
    for (int64_t v = lane; v < row_bytes / 16; v += 32) d[v] = __ldg(s + v);
  } else {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src + t * src_stride);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst + r * row_bytes);
    for (int64_t v = lane; v < row_bytes / 4; v += 32) d[v] = __ldg(s + v);
  }
}

// Transposed gather of per-row scales: dst[kb * cap + r] = src[(sorted_pairs[r] / topk) * src_stride + kb]
// for the rows the align stage filled (0 for padding rows), so the 128 scales of one m-block
// and K block are 512 contiguous bytes (one TMA box). ue8m0: those 512 bytes are the m-block's
// scale-factor atom instead (row r's UE8M0 code, four times, in word (r % 32) * 4 + r / 32).
__global__ void __launch_bounds__(256)
gather_scales_t_kernel(const float* __restrict__ src, int64_t src_stride, int KB,
                       const int32_t* __restrict__ sorted_pairs, const int32_t* __restrict__ block_start, int E,
                       int topk, int64_t cap, bool ue8m0, float* __restrict__ dst) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= cap || r >= (int64_t)__ldg(block_start + E) * kBlockM) return;
  const int pair = __ldg(sorted_pairs + r);
  const float* s = pair >= 0 ? src + (int64_t)(pair / topk) * src_stride : nullptr;
  if (ue8m0) {
    const int64_t w = (r & ~int64_t(127)) + (r & 31) * 4 + ((r >> 5) & 3);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (int kb = 0; kb < KB; ++kb) d[(int64_t)kb * cap + w] = s ? ue8m0x4(__ldg(s + kb)) : 0u;
  } else {
    for (int kb = 0; kb < KB; ++kb) dst[(int64_t)kb * cap + r] = s ? __ldg(s + kb) : 0.f;
  }
}

// [K blocks][rows_cap] fp32 scale table; box = 128 rows of one K block.
bool make_scale_map(CUtensorMap* m, const float* base, int64_t rows_cap, int kblocks) {
  const uint64_t dims[2] = {(uint64_t)rows_cap, (uint64_t)kblocks};
  const uint64_t str[1] = {(uint64_t)rows_cap * 4};
  return make_f32_rows_map(m, base, dims, str, kBlockM);
}

template <int MODE, int STAGES, bool MX>
cudaError_t launch_f8_stages(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msa,
                             const float* b_scale, const int32_t* block_start, int E, int k_red, int n_out, int NB,
                             int64_t rows_cap, void* out, float* out_scale, const int32_t* sorted_pairs, int* status,
                             int max_ctas, cudaStream_t st) {
  auto kern = moe_gemm_fp8_kernel<MODE, STAGES, MX>;
  const int smem = F8Smem<STAGES, MX>::bytes(E);
  cudaFuncAttributes fa;
  cudaError_t err = cudaFuncGetAttributes(&fa, kern);
  if (err != cudaSuccess) return err;
  // setmaxnreg.inc waits for registers the block does not own if the launch holds
  // fewer than 384 x 168: never launch such a build.
  if (fa.numRegs != kF8RegsLaunch) return cudaErrorInvalidConfiguration;
  err = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
  if (err != cudaSuccess) return err;
  const int64_t tiles_cap = (rows_cap / kBlockM) * NB;
  const int ctas = (max_ctas > 0 && max_ctas < num_sms()) ? max_ctas : num_sms();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas, tiles_cap));
  kern<<<grid, kF8Threads, smem, st>>>(ma, mb, msa, b_scale, block_start, E, k_red, n_out, NB, out, out_scale,
                                       rows_cap, sorted_pairs, status);
  return cudaGetLastError();
}

template <int MODE, bool MX>
cudaError_t launch_f8_mx(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msa, const float* b_scale,
                         const int32_t* block_start, int E, int k_red, int n_out, int NB, int64_t rows_cap, void* out,
                         float* out_scale, const int32_t* sorted_pairs, int* status, int max_ctas, cudaStream_t st) {
  constexpr int kMaxSmem = 227 * 1024;
  if (F8Smem<4, MX>::bytes(E) <= kMaxSmem)
    return launch_f8_stages<MODE, 4, MX>(ma, mb, msa, b_scale, block_start, E, k_red, n_out, NB, rows_cap, out,
                                         out_scale, sorted_pairs, status, max_ctas, st);
  if (F8Smem<3, MX>::bytes(E) <= kMaxSmem)
    return launch_f8_stages<MODE, 3, MX>(ma, mb, msa, b_scale, block_start, E, k_red, n_out, NB, rows_cap, out,
                                         out_scale, sorted_pairs, status, max_ctas, st);
  return cudaErrorInvalidValue;
}

template <int MODE>
cudaError_t launch_f8(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msa, const float* b_scale,
                      const int32_t* block_start, int E, int k_red, int n_out, int NB, int64_t rows_cap, void* out,
                      float* out_scale, const int32_t* sorted_pairs, bool ue8m0, int* status, int max_ctas,
                      cudaStream_t st) {
  if (ue8m0)
    return launch_f8_mx<MODE, true>(ma, mb, msa, b_scale, block_start, E, k_red, n_out, NB, rows_cap, out, out_scale,
                                    sorted_pairs, status, max_ctas, st);
  return launch_f8_mx<MODE, false>(ma, mb, msa, b_scale, block_start, E, k_red, n_out, NB, rows_cap, out, out_scale,
                                   sorted_pairs, status, max_ctas, st);
}

}  // namespace

cudaError_t launch_gather_rows(const void* src, int64_t src_stride, int64_t row_bytes, const int32_t* sorted_pairs,
                               const int32_t* block_start, int E, int topk, int64_t cap, void* dst, cudaStream_t st) {
  if (cap == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)ceil_div(cap * 32, 256);
  gather_rows_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint8_t*>(src), src_stride, row_bytes, sorted_pairs,
                                             block_start, E, topk, cap, static_cast<uint8_t*>(dst));
  return cudaGetLastError();
}

cudaError_t launch_gather_scales_t(const float* src, int64_t src_stride, int KB, const int32_t* sorted_pairs,
                                   const int32_t* block_start, int E, int topk, int64_t cap, bool ue8m0, float* dst,
                                   cudaStream_t st) {
  if (cap == 0) return cudaSuccess;
  if (ue8m0 && cap % kBlockM != 0) return cudaErrorInvalidValue;  // atoms cover whole m-blocks
  gather_scales_t_kernel<<<(unsigned)ceil_div(cap, 256), 256, 0, st>>>(src, src_stride, KB, sorted_pairs, block_start,
                                                                       E, topk, cap, ue8m0, dst);
  return cudaGetLastError();
}

cudaError_t launch_fp8_gemm1(const void* xq_sorted, const float* xs_sorted_t, int64_t rows_cap, const void* w1q,
                             const float* w1s, int E, int K, int N, const int32_t* block_start, void* actq,
                             float* acts_t, bool ue8m0, int* status, int max_ctas, cudaStream_t st) {
  CUtensorMap ma, mbm, msa;
  const uint64_t a_dims[2] = {(uint64_t)K, (uint64_t)rows_cap};
  const uint64_t a_str[1] = {(uint64_t)K};
  const uint64_t b_dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)2 * E};
  const uint64_t b_str[2] = {(uint64_t)K, (uint64_t)N * K};
  if (!make_fp8_map(&ma, xq_sorted, 2, a_dims, a_str, kBlockM)) return cudaErrorInvalidValue;
  if (!make_fp8_map(&mbm, w1q, 3, b_dims, b_str, 64)) return cudaErrorInvalidValue;
  if (!make_scale_map(&msa, xs_sorted_t, rows_cap, K / 128)) return cudaErrorInvalidValue;
  return launch_f8<F8_GEMM1>(ma, mbm, msa, w1s, block_start, E, K, N, N / 128, rows_cap, actq, acts_t, nullptr,
                             ue8m0, status, max_ctas, st);
}

cudaError_t launch_fp8_gemm2(const void* actq, const float* acts_t, int64_t rows_cap, const void* w2q,
                             const float* w2s, int E, int K, int N, const int32_t* block_start,
                             const int32_t* sorted_pairs, void* y_slots, bool ue8m0, int* status, int max_ctas,
                             cudaStream_t st) {
  CUtensorMap ma, mbm, msa;
  const uint64_t a_dims[2] = {(uint64_t)N, (uint64_t)rows_cap};
  const uint64_t a_str[1] = {(uint64_t)N};
  const uint64_t b_dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)E};
  const uint64_t b_str[2] = {(uint64_t)N, (uint64_t)K * N};
  if (!make_fp8_map(&ma, actq, 2, a_dims, a_str, kBlockM)) return cudaErrorInvalidValue;
  if (!make_fp8_map(&mbm, w2q, 3, b_dims, b_str, kF8BN)) return cudaErrorInvalidValue;
  if (!make_scale_map(&msa, acts_t, rows_cap, N / 128)) return cudaErrorInvalidValue;
  return launch_f8<F8_GEMM2>(ma, mbm, msa, w2s, block_start, E, N, K, (int)ceil_div(K, kF8BN), rows_cap, y_slots,
                             nullptr, sorted_pairs, ue8m0, status, max_ctas, st);
}

}  // namespace moe

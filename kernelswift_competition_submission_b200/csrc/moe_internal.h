// Internal launch helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/moe_b200.h"

namespace moe {

constexpr int kBlockM = 128;  // rows per m-block of the grouped GEMMs (one TMEM lane per row)

// Metadata of the align stage. counts, cursor and done must be zero before the
// launch; launch_align zeroes them itself.
struct AlignMeta {
  int32_t* counts;       // [E]     pairs per expert
  int32_t* cursor;       // [E]     scratch: rows handed out per expert
  int32_t* block_start;  // [E + 1] prefix sum of ceil(counts / block_m)
  int32_t* done;         // [1]     scratch: CTAs finished counting
};
// Contiguous layout used by the fused path: [counts | cursor | done | block_start];
// the first 2E + 1 ints are the ones zeroed before each launch.
inline int64_t align_meta_ints(int E) { return 3 * (int64_t)E + 2; }
inline AlignMeta align_meta_contiguous(int32_t* meta, int E) {
  return AlignMeta{meta, meta + E, meta + 2 * E + 1, meta + 2 * E};
}

// Launches the align stage. When x_src != nullptr the scatter also copies each
// pair's token row of `row_bytes` bytes from x_src into x_sorted at the pair's
// padded row (x_sorted row pitch = row_bytes).
// zero_meta = false: the caller has zeroed counts, cursor and done on `st` already.
cudaError_t launch_align(const int32_t* topk_ids, int64_t num_pairs, int topk, int E, int block_m, AlignMeta m,
                         bool meta_contiguous, int32_t* sorted_pairs, int64_t sorted_capacity, const void* x_src,
                         void* x_sorted, int64_t row_bytes, cudaStream_t st, bool zero_meta = true);

// Weighted sum over the topk slots: out[t] = sum_j w[t, j] * y[t * topk + j]   (elem = bf16 / fp16).
// Slots whose expert id is outside [0, E) contribute nothing (as in the reference's expert loop).
cudaError_t launch_combine(int dtype, const void* y_slots, const float* topk_weights, const int32_t* topk_ids,
                           int64_t M, int topk, int E, int K, void* out, cudaStream_t st);

// Grouped GEMMs, one CTA per tile (sm_100a tcgen05.mma.cta_group::1, token-major 128 x 256
// tiles). Rows come in m-blocks of kBlockM grouped by expert (align with block_m = kBlockM;
// block_start read on the device).
// max_ctas: persistent grid size limit (0 = one CTA per SM).
cudaError_t launch_gemm1_silu(int dtype, const void* x_sorted, int64_t rows_cap, const void* w1, int E, int K, int N,
                              const int32_t* block_start, void* act, int* status, int max_ctas, cudaStream_t st);
// GEMM1 with its A rows gathered from the token rows (x, row pitch x_ld elements): row r
// of the expert-sorted order is token sorted_pairs[r] / topk, padding rows (-1) are zeros.
// No expert-sorted copy of the tokens is needed.
cudaError_t launch_gemm1_gather(int dtype, const void* x, int64_t x_ld, int topk, const int32_t* sorted_pairs,
                               int64_t rows_cap, const void* w1, int E, int K, int N, const int32_t* block_start,
                               void* act, int* status, int max_ctas, cudaStream_t st);
cudaError_t launch_gemm2_scatter(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                                 const int32_t* block_start, const int32_t* sorted_pairs, int64_t num_pairs,
                                 void* y_slots, int* status, int max_ctas, cudaStream_t st);

// Down GEMM with the top-k combine fused into its epilogue: slot rows go to y_slots
// ([M * topk, K], as launch_gemm2_scatter), and the warp that stores a token's last
// valid slot of an n-block writes out[t, n-block] = sum_j topk_weights[t, j] * y[t*topk+j]
// (fp32, slot order: the bits of launch_combine). arrivals [M, ceil(K / gemm2_block_n(K))]
// must be zero: launch_combine_prep does that and writes the rows of tokens without a
// valid slot.
int gemm2_block_n(int K);
cudaError_t launch_gemm2_combine(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                                 const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots,
                                 const float* topk_weights, const int32_t* topk_ids, int topk, int32_t* arrivals,
                                 void* out, int* status, int max_ctas, cudaStream_t st);
// The same, with each completed row returned into its source rank's arena over peer memory
// (the expert-parallel layer): received row t = src * cap + r goes to back_x row me * cap + r
// of rank src, whose back flag [me] is raised (= seq) when all of its rows are in; see
// CombineArgs in moe_gemm.cu. arrivals [M, NB] and src_done [world] must be zero.
cudaError_t launch_gemm2_return(int dtype, const void* act, int64_t rows_cap, const void* w2, int E, int K, int N,
                                const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots,
                                const float* recv_w, const int32_t* recv_id, int topk, int32_t* arrivals,
                                const int64_t* peer_base, const int32_t* own_counts, int32_t* src_done,
                                int64_t back_off, int64_t flag_off, int64_t cap, int me, int world, uint32_t seq,
                                int* status, int max_ctas, cudaStream_t st);
cudaError_t launch_combine_prep(const int32_t* topk_ids, int64_t M, int topk, int E, int K, int32_t* arrivals,
                                int64_t n_arrivals, int32_t* zero_ints, int n_zero, void* out, cudaStream_t st);

// out[t] = sum over d with tok_rows[t, d] >= 0 of back[tok_rows[t, d]] (fp32); when `status`
// is non-null and holds a failure code, every output element is NaN instead.
cudaError_t launch_ep_combine(int dtype, const void* back, const int32_t* tok_rows, int64_t M, int K, int world,
                              void* out, const int* status, cudaStream_t st);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (function, device) and size.
cudaError_t ensure_smem_limit(const void* func, int bytes);

// Tensor maps (cuTensorMapEncodeTiled), cached by address, shape, strides and box.
bool make_kmajor_map(CUtensorMap* m, int dtype, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, uint32_t box_rows);

bool make_fp8_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                  uint32_t box_rows);

// FP8 path: tcgen05.mma.kind::f8f6f4 per 128-wide K block, fp32 block-scale
// promotion in the epilogue. Row scales are [K blocks][rows_cap] tables (the
// transpose of the per-row layout). GEMM1 writes e4m3 act rows + their scales
// (SiLU*mul quantised in the epilogue); GEMM2 writes bf16 pair slots.
bool make_f32_rows_map(CUtensorMap* m, const float* base, const uint64_t* dims, const uint64_t* strides_bytes,
                       uint32_t box_rows);
// max_ctas: persistent grid size limit (0 = one CTA per SM).
// With ue8m0 (every scale a power of two) the GEMMs run kind::mxf8f6f4.block_scale
// instead: row scales are then UE8M0 atom tables (launch_gather_scales_t with ue8m0),
// the weight scales' exponents become the B scale factors, and GEMM1 writes act's
// scales as such a table too.
cudaError_t launch_fp8_gemm1(const void* xq_sorted, const float* xs_sorted_t, int64_t rows_cap, const void* w1q,
                             const float* w1s, int E, int K, int N, const int32_t* block_start, void* actq,
                             float* acts_t, bool ue8m0, int* status, int max_ctas, cudaStream_t st);
cudaError_t launch_fp8_gemm2(const void* actq, const float* acts_t, int64_t rows_cap, const void* w2q,
                             const float* w2s, int E, int K, int N, const int32_t* block_start,
                             const int32_t* sorted_pairs, void* y_slots, bool ue8m0, int* status, int max_ctas,
                             cudaStream_t st);
// dst[kb * cap + r] = src[(sorted_pairs[r] / topk) * src_stride + kb] for the rows the align
// stage filled (src_stride in floats between token rows). With ue8m0 the 128 entries of an
// m-block and K block form the scale-factor atom of tcgen05's block-scaled MMA instead: the
// word of row r at (r / 128) * 128 + (r % 32) * 4 + (r % 128) / 32, holding the scale's UE8M0
// code in all four bytes (one per 32-wide K chunk); 0 for padding rows.
cudaError_t launch_gather_scales_t(const float* src, int64_t src_stride, int KB, const int32_t* sorted_pairs,
                                   const int32_t* block_start, int E, int topk, int64_t cap, bool ue8m0, float* dst,
                                   cudaStream_t st);
// dst[r] = row_bytes bytes of src at token row sorted_pairs[r] / topk (src_stride bytes apart),
// for the rows the align stage filled; dst rows are row_bytes apart.
cudaError_t launch_gather_rows(const void* src, int64_t src_stride, int64_t row_bytes, const int32_t* sorted_pairs,
                               const int32_t* block_start, int E, int topk, int64_t cap, void* dst, cudaStream_t st);

// FP8 GEMMs for decode-sized batches (moe_gemm_fp8_swap.cu): 128 weight rows x 32 tokens
// per tile, with the expert's row counts (align `counts`) choosing the tiles on the device.
// Same inputs and outputs as launch_fp8_gemm1 / launch_fp8_gemm2. The FP8 path takes them
// when the experts average no more than kFp8SwapMaxRowsPerExpert rows (fp8_use_swap).
constexpr int64_t kFp8SwapMaxRowsPerExpert = 16;
bool fp8_use_swap(int64_t num_pairs, int E);
// pow2_act: act's scales rounded up to powers of two (the UE8M0 recipe).
cudaError_t launch_fp8_swap_gemm1(const void* xq_sorted, const float* xs_sorted_t, int64_t rows_cap,
                                  int64_t num_pairs, const void* w1q, const float* w1s, int E, int K, int N,
                                  const int32_t* counts, const int32_t* block_start, void* actq, float* acts_t,
                                  bool pow2_act, int* status, int max_ctas, cudaStream_t st);
cudaError_t launch_fp8_swap_gemm2(const void* actq, const float* acts_t, int64_t rows_cap, int64_t num_pairs,
                                  const void* w2q, const float* w2s, int E, int K, int N, const int32_t* counts,
                                  const int32_t* block_start, const int32_t* sorted_pairs, void* y_slots, int* status,
                                  int max_ctas, cudaStream_t st);

// Per row, per 128 columns e4m3 quantisation (dtype bf16 / fp16 / fp32 input): row m's codes
// at q + m * ldq (bytes), its K / 128 scales at s + m * lds (floats).
cudaError_t launch_quantize_rows(int dtype, const void* x, int64_t M, int K, uint8_t* q, int64_t ldq, float* s,
                                 int64_t lds, bool pow2, cudaStream_t st);
inline bool scale_fmt_ok(int f) { return f == MOE_FP8_SCALE_FP32 || f == MOE_FP8_SCALE_UE8M0; }

// Packed e4m3 token row (MOE_DTYPE_E4M3_ROW): K codes, then K / 128 fp32 scales, padded to
// a multiple of 16 bytes.
inline int64_t fp8_row_bytes(int K) { return (int64_t)K + ((int64_t)K / 32 + 15) / 16 * 16; }

// Byte offset of the bf16 y slot rows ([M * topk, K]) in the FP8 expert workspace.
size_t fp8_yslots_offset(int64_t M, int E, int topk, int K, int N);

int num_sms();

// Byte offset of the y_slots region ([M * topk, K] slot rows) in the fused workspace.
size_t fused_yslots_offset(int64_t M, int E, int topk, int K, int N);

}  // namespace moe

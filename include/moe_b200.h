/*
 * moe_b200.h — C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * The reference (kernelswift_competition_submission) exposes this path only as
 * Python modules: `grouped_topk/v1/grouped_topk.py` (ModelNew.forward ->
 * _grouped_topk_kernel) and `fused_moe/v1/fused_moe.py` (ModelNew.forward ->
 * _moe_expert_kernel + _moe_reduce_kernel). Each entry point below replaces one
 * of those launches; the Python layer of this project (ctypes) binds them the
 * way the reference's ModelNew binds its Triton kernels.
 *
 * Conventions
 *   - All data pointers are DEVICE pointers on the current CUDA device; sizes
 *     are element counts; `stream` is a cudaStream_t passed as void* (NULL =
 *     legacy default stream).
 *   - Every function returns an int status (MOE_OK = 0). Argument errors are
 *     detected on the host before any launch. Device-side failures (a bounded
 *     wait that gave up) are recorded in the optional `status` word, a device
 *     int the caller zeroes and reads after synchronising.
 *   - No function allocates device memory except moe_p2p_alloc (the peer-memory
 *     arena that other ranks map through CUDA IPC); scratch comes from the caller's
 *     workspace (see moe_fused_workspace_bytes).
 *   - Inputs are never written.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARG 1 /* null pointer, negative size, unknown enum value */
#define MOE_ERR_BAD_SHAPE 2   /* shape outside what the kernels support */
#define MOE_ERR_UNSUPPORTED 3 /* dtype or rule not implemented */
#define MOE_ERR_NOT_SM100 4   /* current device is not compute capability 10.x */
#define MOE_ERR_WORKSPACE 5   /* workspace smaller than required */
#define MOE_ERR_CUDA 6        /* a CUDA runtime call failed */
#define MOE_ERR_TIMEOUT 7     /* a bounded device-side wait gave up */
#define MOE_ERR_SCRATCH_LIMIT 8 /* request exceeds the fixed scratch of moe_align_noalloc */

/* scoring_func */
#define MOE_SCORING_SOFTMAX 0
#define MOE_SCORING_SIGMOID 1
/* group_score_mode */
#define MOE_GROUP_SCORE_MAX 0      /* reference v0 rule: best expert of the group */
#define MOE_GROUP_SCORE_TOP2_SUM 1 /* DeepSeek-V3 rule: sum of the group's two best */
/* element types of hidden_states / w1 / w2 / out */
#define MOE_DTYPE_BF16 0
#define MOE_DTYPE_FP16 1
#define MOE_DTYPE_FP32 2 /* FP8 quantiser inputs only */
/* Packed e4m3 token row (expert-parallel FP8 payload): hidden_size e4m3 codes, then
 * hidden_size / 128 fp32 scales (per token per 128), padded to a multiple of 16 bytes
 * (moe_fp8_row_bytes). Accepted by moe_ep_pack*, moe_p2p_dispatch and
 * moe_p2p_combine_experts_back. */
#define MOE_DTYPE_E4M3_ROW 3

/* Human-readable name of a status code (static string). */
MOE_API const char* moe_status_string(int status);

/* Library ABI version (major * 100 + minor). */
MOE_API int moe_abi_version(void);

/* MOE_OK when the current device is sm_100 (B200/GB200), else MOE_ERR_NOT_SM100
 * or MOE_ERR_CUDA. */
MOE_API int moe_check_device(void);

/*
 * grouped_topk routing.
 * Replaces grouped_topk/v1/grouped_topk.py:210-235 (ModelNew.forward launching
 * _grouped_topk_kernel); the rule is grouped_topk/v0/grouped_topk.py:91-132.
 *
 *   gating_output            fp32 [num_tokens, num_experts], row-major
 *   e_score_correction_bias  fp32 [num_experts] or NULL (NULL = reference v0 rule)
 *   topk_weights (out)       fp32 [num_tokens, topk]
 *   topk_ids (out)           int32 [num_tokens, topk], sorted by score descending,
 *                            ties broken by the lowest expert index
 * Ranking uses scores (+ bias when given); weights are the scores without the
 * bias, renormalised when `renormalize`, then multiplied by
 * routed_scaling_factor. Supports num_experts <= 512, num_expert_group <= 32,
 * topk <= 32 and topk <= topk_group * (num_experts / num_expert_group).
 * The fused_moe routing of fused_moe/v0/fused_moe.py:134-139 is the special
 * case num_expert_group = topk_group = 1, softmax, scale 1.
 */
MOE_API int moe_grouped_topk(const float* gating_output, const float* e_score_correction_bias,
                     int64_t num_tokens, int num_experts, int topk, int renormalize,
                     int num_expert_group, int topk_group, int scoring_func, int group_score_mode,
                     float routed_scaling_factor, float* topk_weights, int32_t* topk_ids,
                     void* stream);

/*
 * Token -> expert align stage (counting sort of (token, slot) pairs).
 * Replaces the per-expert boolean masks of fused_moe/v0/fused_moe.py:143-159
 * and the routing recomputation inside fused_moe/v1/fused_moe.py:182-197.
 *
 *   topk_ids      int32 [num_pairs]   (num_pairs = num_tokens * topk, row-major)
 *   counts (out)  int32 [num_experts]
 *   block_start (out) int32 [num_experts + 1]  prefix sum of ceil(count / block_m)
 *   sorted_pairs (out) int32 [sorted_capacity]  pair id per padded row, -1 in padding;
 *                 rows of expert e are [block_start[e] * block_m, block_start[e+1] * block_m)
 *   scratch       int32 [num_experts + 1] device scratch (overwritten)
 * sorted_capacity must be >= moe_align_capacity(num_pairs, num_experts, block_m).
 * Order of pairs inside one expert's segment is unspecified.
 */
MOE_API int64_t moe_align_capacity(int64_t num_pairs, int num_experts, int block_m);
MOE_API int moe_align(const int32_t* topk_ids, int64_t num_pairs, int num_experts, int block_m,
              int32_t* counts, int32_t* block_start, int32_t* sorted_pairs, int64_t sorted_capacity,
              int32_t* scratch, void* stream);

/*
 * moe_align_noalloc: moe_align for callers that cannot allocate device memory.
 * No counterpart in the reference (its align step is the per-expert Python
 * loop of fused_moe/v0/fused_moe.py:155-159, which allocates freely).
 *
 * Who needs it: a caller whose device memory is owned by someone else, e.g.
 * an inference engine that reserves nearly all of HBM up front for its own
 * pools and does not allow side allocations, or a foreign-language binding
 * that has no handle on the host framework's allocator, cannot produce the
 * `scratch` buffer moe_align asks for. This entry point needs only the
 * inputs and outputs: its scratch (one int per expert plus one counter) is a
 * fixed array inside the library.
 *
 * Same arguments, outputs and ordering rules as moe_align, minus `scratch`.
 * Limits and behaviour:
 *   - num_experts <= MOE_NOALLOC_MAX_EXPERTS (1024); larger requests return
 *     MOE_ERR_SCRATCH_LIMIT before anything is enqueued.
 *   - The scratch array (4100 bytes) is held by every GPU that loads this
 *     library until the process exits.
 *   - The first call on a device looks up the array's device address with
 *     cudaGetSymbolAddress (with that device current) and caches it; make that
 *     first call before any stream capture.
 *   - All calls share the one array. Each call zeroes what must start at zero
 *     on its own stream, but calls that overlap on the GPU (different streams,
 *     not ordered by events) race on it: serialise them.
 *   - Calls no cudaMalloc, cudaFree or other allocating routine.
 */
#define MOE_NOALLOC_MAX_EXPERTS 1024
MOE_API int moe_align_noalloc(const int32_t* topk_ids, int64_t num_pairs, int num_experts, int block_m,
                              int32_t* counts, int32_t* block_start, int32_t* sorted_pairs,
                              int64_t sorted_capacity, void* stream);

/*
 * Expert computation of fused_moe for given routing.
 * Replaces fused_moe/v1/fused_moe.py:305-341 (ModelNew.forward after routing:
 * _moe_expert_kernel + _moe_reduce_kernel); the math is
 * fused_moe/v0/fused_moe.py:141-167:
 *   out[t] = sum_j topk_weights[t, j] * (silu(x[t] W1g^T) * (x[t] W1u^T)) W2^T,
 *   with expert e = topk_ids[t, j], W1g = w1[e, :N, :], W1u = w1[e, N:, :], W2 = w2[e].
 *
 *   dtype          MOE_DTYPE_BF16 or MOE_DTYPE_FP16 (x, w1, w2, out)
 *   hidden_states  [num_tokens, hidden_size]
 *   w1             [num_experts, 2 * intermediate_size, hidden_size]
 *   w2             [num_experts, hidden_size, intermediate_size]
 *   topk_weights   fp32 [num_tokens, topk]
 *   topk_ids       int32 [num_tokens, topk], values in [0, num_experts)
 *   out            [num_tokens, hidden_size]
 *   workspace      device buffer of >= moe_fused_workspace_bytes(...) bytes, 256-B aligned
 *   status         optional device int (NULL allowed); a device-side timeout writes
 *                  MOE_ERR_TIMEOUT there
 * Requires hidden_size % 64 == 0 and intermediate_size % 64 == 0, all pointers
 * 16-byte aligned. GEMMs run on tcgen05 tensor cores with TMA-fed operands and
 * TMEM accumulators; SiLU*mul is fused into the gate/up GEMM epilogue.
 */
MOE_API size_t moe_fused_workspace_bytes(int64_t num_tokens, int num_experts, int topk, int hidden_size,
                                 int intermediate_size);
MOE_API int moe_fused_experts(int dtype, const void* hidden_states, const void* w1, const void* w2,
                      const float* topk_weights, const int32_t* topk_ids, int64_t num_tokens,
                      int num_experts, int topk, int hidden_size, int intermediate_size, void* out,
                      void* workspace, size_t workspace_bytes, int* status, void* stream);

/*
 * The stages of moe_fused_experts as separate calls on the same workspace
 * (same arguments as moe_fused_experts), in this order:
 *   moe_expert_align_gather  align stage + gather of each pair's token row into
 *                            expert-sorted order (workspace)
 *   moe_expert_gemm1         tcgen05 gate/up GEMM, SiLU*mul epilogue -> act (workspace)
 *   then either
 *   moe_expert_gemm2_combine tcgen05 down GEMM with the top-k weighted sum fused into
 *                            its epilogue -> out (replaces fused_moe/v0/fused_moe.py:163-167
 *                            and the reduce kernel fused_moe/v1/fused_moe.py:221-252)
 *   or
 *   moe_expert_gemm2         tcgen05 down GEMM, per-pair rows -> slot buffer (workspace)
 *   moe_expert_combine       top-k weighted sum of the slot rows -> out
 * Both endings give the same bits: the fused epilogue sums a token's slot rows in slot
 * order in fp32, exactly as moe_expert_combine does, once all of them are stored. The
 * separate combine is the faster one at prefill sizes (a token's last slot arrives with
 * its highest-numbered expert, so the fused sums bunch up in the GEMM's last tiles);
 * moe_fused_experts(...) runs align_gather, gemm1, gemm2 and combine (max_ctas = 0).
 * They exist so a caller can interleave its own work (events, communication)
 * between stages. max_ctas limits the persistent GEMM grid (0 = one CTA per
 * SM) so that work on other streams, e.g. collectives, can run beside it.
 */
MOE_API int moe_expert_align_gather(int dtype, const void* hidden_states, const int32_t* topk_ids,
                                    int64_t num_tokens, int num_experts, int topk, int hidden_size,
                                    int intermediate_size, void* workspace, size_t workspace_bytes,
                                    void* stream);
/* The same expert path without the expert-sorted copy of the token rows (the workspace
 * region the gather fills is left untouched, so a caller may size it away):
 * moe_expert_align (the align stage alone), then moe_expert_gemm1_gather, the gate/up
 * GEMM reading each A row straight from hidden_states (token sorted_pairs[r] / topk) with
 * cp.async into the tensor-core layout, then either GEMM2 ending. Same bits as
 * align_gather + gemm1; slower at prefill sizes (the tensor core waits on the cp.async
 * row copies), so it is the choice for tight memory rather than for speed. */
MOE_API int moe_expert_align(const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                             int hidden_size, int intermediate_size, void* workspace, size_t workspace_bytes,
                             void* stream);
MOE_API int moe_expert_gemm1_gather(int dtype, const void* hidden_states, const void* w1, int64_t num_tokens,
                                    int num_experts, int topk, int hidden_size, int intermediate_size,
                                    void* workspace, size_t workspace_bytes, int* status, int max_ctas,
                                    void* stream);
MOE_API int moe_expert_gemm1(int dtype, const void* w1, int64_t num_tokens, int num_experts, int topk,
                             int hidden_size, int intermediate_size, void* workspace,
                             size_t workspace_bytes, int* status, int max_ctas, void* stream);
MOE_API int moe_expert_gemm2(int dtype, const void* w2, int64_t num_tokens, int num_experts, int topk,
                             int hidden_size, int intermediate_size, void* workspace,
                             size_t workspace_bytes, int* status, int max_ctas, void* stream);
MOE_API int moe_expert_gemm2_combine(int dtype, const void* w2, const float* topk_weights,
                                     const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                                     int hidden_size, int intermediate_size, void* out, void* workspace,
                                     size_t workspace_bytes, int* status, int max_ctas, void* stream);
MOE_API int moe_expert_combine(int dtype, const float* topk_weights, const int32_t* topk_ids,
                               int64_t num_tokens, int num_experts, int topk, int hidden_size,
                               int intermediate_size, void* out, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * FP8 (e4m3) block quantisation, the w8a8 recipe of the FP8 layer configuration
 * (no counterpart in the reference, whose path is fp16/bf16/fp32 only):
 *   scale = amax(|block|) / 448 (1.0 for an all-zero block), q = e4m3(x / scale),
 *   rounded to nearest even, saturating at +-448.
 * scale_fmt MOE_FP8_SCALE_FP32 keeps that fp32 scale; MOE_FP8_SCALE_UE8M0 rounds it
 * up to the next power of two (an exact UE8M0 code, the block-scale format of
 * tcgen05's kind::mxf8f6f4 MMA).
 *   moe_quantize_rows_fp8    per row, per 128 columns (activations, per token):
 *                            x [num_rows, cols] -> q uint8 [num_rows, cols],
 *                            scales fp32 [num_rows, cols / 128]
 *   moe_quantize_blocks_fp8  per 128 x 128 block of each [rows, cols] matrix
 *                            (expert weights): w [batch, rows, cols] -> q uint8
 *                            [batch, rows, cols], scales fp32 [batch, rows/128, cols/128]
 * dtype: MOE_DTYPE_BF16, MOE_DTYPE_FP16 or MOE_DTYPE_FP32. cols (and rows) % 128 == 0.
 */
#define MOE_FP8_SCALE_FP32 0
#define MOE_FP8_SCALE_UE8M0 1
MOE_API int moe_quantize_rows_fp8(int dtype, const void* x, int64_t num_rows, int cols, void* q,
                                  float* scales, int scale_fmt, void* stream);
MOE_API int moe_quantize_blocks_fp8(int dtype, const void* w, int64_t batch, int rows, int cols, void* q,
                                    float* scales, int scale_fmt, void* stream);

/*
 * Expert computation of the FP8 w8a8 configuration (DeepSeek-V3 recipe; no
 * counterpart in the reference, which has no FP8 code): the math of
 * moe_fused_experts on dequantised operands.
 *   hidden_states  bf16 [num_tokens, hidden_size]; quantised here per token per 128
 *   w1_q, w1_scale e4m3 [E, 2N, K] and fp32 [E, 2N/128, K/128] (moe_quantize_blocks_fp8)
 *   w2_q, w2_scale e4m3 [E, K, N]  and fp32 [E, K/128, N/128]
 *   out            bf16 [num_tokens, hidden_size]
 * The SiLU*mul output is quantised per row per 128 before the down projection.
 * scale_fmt names the scales of the weights, and the tokens and SiLU*mul rows are
 * quantised the same way:
 *   MOE_FP8_SCALE_FP32   any fp32 scales: both GEMMs run tcgen05.mma.kind::f8f6f4,
 *                        one MMA chain per 128-wide K block, and promote each
 *                        block's fp32 partial sums into the totals with its row
 *                        and weight scales.
 *   MOE_FP8_SCALE_UE8M0  the caller promises every weight scale is a power of two
 *                        (moe_quantize_blocks_fp8 with MOE_FP8_SCALE_UE8M0): at
 *                        prefill sizes the GEMMs run kind::mxf8f6f4.block_scale,
 *                        the tensor cores apply the scales, and one MMA chain
 *                        covers the whole K (no promotion).
 * Requires hidden_size % 128 == 0 and intermediate_size % 128 == 0.
 */
MOE_API size_t moe_fused_workspace_bytes_fp8(int64_t num_tokens, int num_experts, int topk, int hidden_size,
                                             int intermediate_size);
MOE_API int moe_fused_experts_fp8(const void* hidden_states, const void* w1_q, const float* w1_scale,
                                  const void* w2_q, const float* w2_scale, const float* topk_weights,
                                  const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                                  int hidden_size, int intermediate_size, int scale_fmt, void* out,
                                  void* workspace, size_t workspace_bytes, int* status, void* stream);

/*
 * FP8 expert path from token rows quantised elsewhere (the expert-parallel FP8
 * payload, MOE_DTYPE_E4M3_ROW): row t is `rows + t * row_stride`, its hidden_size
 * e4m3 codes followed by hidden_size / 128 fp32 scales (powers of two with
 * MOE_FP8_SCALE_UE8M0, as the weights'). row_stride >=
 * moe_fp8_row_bytes(hidden_size) and a multiple of 16. Same workspace as
 * moe_fused_experts_fp8. topk_ids may hold -1 (slot skipped). With out == NULL
 * the combine is left out and the per-slot rows stay in the workspace, for
 * moe_p2p_combine_experts_back (dtype MOE_DTYPE_E4M3_ROW); topk_weights may then
 * be NULL. max_ctas limits the GEMMs' persistent grids (0 = one CTA per SM).
 *
 *   moe_fp8_row_bytes              bytes of one packed row: hidden_size + hidden_size / 32,
 *                                  rounded up to 16 (-1 unless hidden_size % 128 == 0)
 *   moe_quantize_rows_fp8_packed   x [num_rows, cols] (bf16 / fp16 / fp32) -> packed rows
 *                                  [num_rows, moe_fp8_row_bytes(cols)], the quantisation of
 *                                  moe_quantize_rows_fp8 (padding bytes are left as they are)
 */
MOE_API int64_t moe_fp8_row_bytes(int hidden_size);
MOE_API int moe_quantize_rows_fp8_packed(int dtype, const void* x, int64_t num_rows, int cols, void* rows,
                                         int scale_fmt, void* stream);
MOE_API int moe_fused_experts_fp8_rows(const void* rows, int64_t row_stride, const void* w1_q, const float* w1_scale,
                                       const void* w2_q, const float* w2_scale, const float* topk_weights,
                                       const int32_t* topk_ids, int64_t num_tokens, int num_experts, int topk,
                                       int hidden_size, int intermediate_size, int scale_fmt, void* out,
                                       void* workspace, size_t workspace_bytes, int max_ctas, int* status,
                                       void* stream);

/*
 * Expert-parallel dispatch / combine (the reference has no multi-device code;
 * these serve the expert-parallel form of the layer, experts split evenly over
 * `world` ranks: rank d owns experts [d * experts_per_rank, (d+1) * experts_per_rank)).
 * A token is sent once to each rank owning one of its top-k experts.
 *
 *   moe_ep_send_capacity  upper bound on rows one rank sends: num_tokens * min(topk, world)
 *   moe_ep_plan           per-destination row counts: offsets int32 [world + 1] (row
 *                         offset of each destination block in the send buffer) and
 *                         counts int64 [world] (all-to-all split sizes);
 *                         scratch int32 [2 * world + 1]
 *   moe_ep_pack           copies each token's hidden row into its destination blocks of
 *                         send_x [capacity, hidden_size]; send_meta int32 [capacity, 2*topk]
 *                         holds the k expert ids in the destination's numbering (-1 when
 *                         the destination does not own that slot's expert) followed by the
 *                         k weights as fp32 bits; tok_rows int32 [num_tokens, world] records
 *                         the send row of each (token, destination) or -1. Same scratch
 *                         and offsets as the moe_ep_plan call before it, same stream.
 *   moe_ep_combine        out[t] = sum over d with tok_rows[t, d] >= 0 of
 *                         returned_rows[tok_rows[t, d]] (fp32 accumulation)
 * Requires world <= 64, topk <= 32, hidden_size % 8 == 0.
 */
MOE_API int64_t moe_ep_send_capacity(int64_t num_tokens, int topk, int world);
MOE_API int moe_ep_plan(const int32_t* topk_ids, int64_t num_tokens, int topk, int experts_per_rank,
                        int world, int32_t* scratch, int32_t* offsets, int64_t* counts, void* stream);
MOE_API int moe_ep_pack(int dtype, const void* hidden_states, const int32_t* topk_ids,
                        const float* topk_weights, int64_t num_tokens, int hidden_size, int topk,
                        int experts_per_rank, int world, int32_t* scratch, const int32_t* offsets,
                        void* send_x, int32_t* send_meta, int32_t* tok_rows, void* stream);
MOE_API int moe_ep_combine(int dtype, const void* returned_rows, const int32_t* tok_rows,
                           int64_t num_tokens, int hidden_size, int world, void* out, void* stream);

/* Router GEMM fused with grouped_topk (no reference counterpart: the reference's
 * path starts from the logits, grouped_topk/v0/grouped_topk.py:93-94).
 *   logits_out fp32 [num_tokens, 256] = hidden_states [num_tokens, hidden_size] .
 *   w_gate [256, hidden_size]^T (bf16 or fp16, dtype MOE_DTYPE_*, fp32 accumulation),
 *   then the moe_grouped_topk rule on those logits into topk_weights / topk_ids.
 * num_experts must be 256, hidden_size % 64 == 0, and when groups are masked each
 * group must span a power-of-two number of 8-expert lanes. scratch: int32
 * [moe_router_scratch_ints(num_tokens)] per-call counters. logits_out is written
 * (and zeroed first when an m-block's K range is split over several CTAs). */
MOE_API int64_t moe_router_scratch_ints(int64_t num_tokens);
MOE_API int moe_router_grouped_topk(int dtype, const void* hidden_states, const void* w_gate, const float* bias,
                                    int64_t num_tokens, int num_experts, int hidden_size, int topk,
                                    int renormalize, int num_expert_group, int topk_group, int scoring_func,
                                    int group_score_mode, float routed_scaling_factor, float* logits_out,
                                    float* topk_weights, int32_t* topk_ids, int32_t* scratch, int* status,
                                    void* stream);

/* Expert-parallel dispatch / combine over NVLink peer memory (no reference counterpart;
 * decode-sized batches). Each rank allocates one arena (moe_p2p_alloc: moe_p2p_arena_bytes
 * of device memory with its flags and counts zeroed and its id rows set to -1, and its
 * 64-byte CUDA IPC handle), opens every other rank's handle (moe_p2p_open) and keeps
 * the world base pointers in a device int64 array `peer_bases` (its own at index me).
 * Per step with sequence number seq (1, 2, ...): moe_p2p_signal(which 0: ready),
 * moe_p2p_dispatch (waits for every rank's ready, writes token rows / ids / weights into
 * the destination ranks' arenas, then their disp flags), moe_p2p_wait(which 1) before the
 * local expert path over the world * cap received rows (recv_x, recv_id, recv_w at
 * moe_p2p_arena_offsets[4..6]), moe_p2p_combine_back (returns the partial rows, then back
 * flags), moe_p2p_wait(which 2), then moe_p2p_reduce (or moe_ep_combine over back_x,
 * offset [7]) with the tok_rows the dispatch wrote. scratch: int32 [2 * world + 1] zeroed
 * once (dispatch), int32 [1] zeroed once (combine_back).
 * Failure: waits are bounded (2 s); one that gives up records MOE_ERR_TIMEOUT in `status`.
 * Every moe_p2p_* kernel reads `status` first and does nothing once it is set (no waits,
 * no peer stores, no flags), and moe_p2p_reduce then writes NaN rows, so a failed step
 * never returns another step's rows. The arenas must then be rebuilt on every rank
 * (free, alloc, exchange handles) with the status word zeroed before the next step.
 * offsets[9]: ready, disp, back, counts, recv_x, recv_id, recv_w, back_x, total. */
MOE_API int64_t moe_p2p_arena_bytes(int world, int64_t cap, int hidden_size, int topk);
MOE_API int moe_p2p_arena_offsets(int world, int64_t cap, int hidden_size, int topk, int64_t* offsets);
MOE_API int moe_p2p_alloc(int world, int64_t cap, int hidden_size, int topk, void** base, void* ipc_handle);
MOE_API int moe_p2p_open(const void* ipc_handle, void** base);
MOE_API int moe_p2p_close(void* base);
MOE_API int moe_p2p_free(void* base);
MOE_API int moe_p2p_signal(const int64_t* peer_bases, int world, int me, int which, int64_t cap, int hidden_size,
                           int topk, uint32_t seq, int* status, void* stream);
MOE_API int moe_p2p_wait(const void* own_base, int world, int which, int64_t cap, int hidden_size, int topk,
                         uint32_t seq, int* status, void* stream);
MOE_API int moe_p2p_dispatch(int dtype, const void* hidden_states, const int32_t* topk_ids,
                             const float* topk_weights, int64_t num_tokens, int hidden_size, int topk,
                             int experts_per_rank, int world, int me, int64_t cap, const int64_t* peer_bases,
                             const void* own_base, uint32_t seq, int32_t* scratch, int32_t* tok_rows, int* status,
                             void* stream);
/* the expert path's top-k combine fused with moe_p2p_combine_back: after moe_expert_gemm2
 * over the world * cap received rows, sums each valid row's slots from the fused workspace
 * (same M = world * cap, E, topk, K, N as the stages) and stores it into its source's back_x.
 * FP8 payloads (dispatch with MOE_DTYPE_E4M3_ROW; rows at pitch moe_fp8_row_bytes in recv_x):
 * the expert path is moe_fused_experts_fp8_rows with out == NULL, this call then takes
 * dtype MOE_DTYPE_E4M3_ROW and its workspace, and returns bf16 rows. */
MOE_API int moe_p2p_combine_experts_back(int dtype, const void* workspace, int num_experts, int hidden_size,
                                         int intermediate_size, int topk, int world, int me, int64_t cap,
                                         const int64_t* peer_bases, const void* own_base, uint32_t seq,
                                         int32_t* scratch, int* status, void* stream);
/* The down GEMM of the local expert path fused with the combine and the return trip: after
 * moe_expert_align_gather and moe_expert_gemm1 over the world * cap received rows (same
 * workspace, M = world * cap), the epilogue of the down GEMM sums each received row's slots
 * of one n-block once all of them are stored (the bits of moe_p2p_combine_experts_back) and
 * stores the sum straight into the source rank's back_x region `me` over NVLink, so the
 * return overlaps the tensor-core work; the back flag [me] of a source is raised when its
 * last row is in, and at once for a source that sent nothing this step. scratch: int32
 * [world] (zeroed by the call). bf16 / fp16 rows only; the FP8 path keeps
 * moe_p2p_combine_experts_back. */
MOE_API int moe_p2p_expert_gemm2_return(int dtype, const void* w2, void* workspace, size_t workspace_bytes,
                                        int num_experts, int hidden_size, int intermediate_size, int topk,
                                        int world, int me, int64_t cap, const int64_t* peer_bases,
                                        const void* own_base, uint32_t seq, int32_t* scratch, int* status,
                                        int max_ctas, void* stream);
/* copy of the received expert ids [world * cap, topk] (statistics, tests) */
MOE_API int moe_p2p_copy_recv_ids(const void* own_base, int world, int64_t cap, int hidden_size, int topk,
                                  int32_t* dst, void* stream);
MOE_API int moe_p2p_combine_back(int dtype, const void* partial, int hidden_size, int topk, int world, int me,
                                 int64_t cap, const int64_t* peer_bases, const void* own_base, uint32_t seq,
                                 int32_t* scratch, int* status, void* stream);
/* out[t] = sum of the rows the experts' ranks returned for token t (back_x rows named by
 * tok_rows, fp32 accumulation); NaN rows when `status` holds a failure code. */
MOE_API int moe_p2p_reduce(int dtype, const void* own_base, const int32_t* tok_rows, int64_t num_tokens,
                           int hidden_size, int topk, int world, int64_t cap, void* out, const int* status,
                           void* stream);

/* Expert placement by table instead of contiguous ranges: expert_map int32 [num_experts]
 * holds (rank << 16) | local_id for every expert, so a rank can keep replicas of hot
 * experts and route their pairs to itself (the map is then per rank). Otherwise the
 * same as moe_ep_plan / moe_ep_pack (no reference counterpart: load placement for
 * skewed routing). */
MOE_API int moe_ep_plan_mapped(const int32_t* topk_ids, int64_t num_tokens, int topk, int num_experts,
                               const int32_t* expert_map, int world, int32_t* scratch, int32_t* offsets,
                               int64_t* counts, void* stream);
MOE_API int moe_ep_pack_mapped(int dtype, const void* hidden_states, const int32_t* topk_ids,
                               const float* topk_weights, int64_t num_tokens, int hidden_size, int topk,
                               int num_experts, const int32_t* expert_map, int world, int32_t* scratch,
                               const int32_t* offsets, void* send_x, int32_t* send_meta, int32_t* tok_rows,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */

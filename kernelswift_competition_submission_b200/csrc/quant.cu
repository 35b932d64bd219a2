// FP8 (e4m3) block quantisation (the reference has no FP8 code; this is the
// DeepSeek-V3 w8a8 recipe the FP8 configuration of the layer defines):
//   scale = amax(|block|) / 448 (1 for an all-zero block), q = e4m3(x / scale),
//   round to nearest even, saturating at +-448 (__NV_SATFINITE).
// With MOE_FP8_SCALE_UE8M0 the scale is rounded up to a power of two (the UE8M0
// block-scale format of tcgen05's kind::mxf8f6f4 MMA; DeepSeek's scale format on
// Blackwell), so x / scale is exact before the e4m3 rounding.
// quantize_rows_kernel    one warp per (row, 128 columns): each lane holds 4
//                         values, warp max, one 128-byte coalesced store.
// quantize_blocks_kernel  one CTA per 128 x 128 block (weights, done once).
#include "common.cuh"
#include "moe_internal.h"

#include <cuda_fp8.h>

namespace moe {
namespace {

template <typename T> __device__ __forceinline__ float load_f(const T* p) { return (float)*p; }
template <> __device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <> __device__ __forceinline__ float load_f<__half>(const __half* p) { return __half2float(*p); }

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

template <typename T>
__global__ void __launch_bounds__(256)
quantize_rows_kernel(const T* __restrict__ x, int64_t M, int K, uint8_t* __restrict__ q, int64_t ldq,
                     float* __restrict__ s, int64_t lds, bool pow2) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nb = K / 128;
  if (wid >= M * nb) return;
  const int64_t row = wid / nb;
  const int b = (int)(wid - row * nb);
  const T* src = x + row * K + b * 128 + lane * 4;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = load_f(src + i);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float sc = fp8_block_scale(amax, pow2);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) packed |= (uint32_t)to_e4m3(v[i] / sc) << (8 * i);
  reinterpret_cast<uint32_t*>(q + row * ldq + b * 128)[lane] = packed;
  if (lane == 0) s[row * lds + b] = sc;
}

template <typename T>
__global__ void __launch_bounds__(256)
quantize_blocks_kernel(const T* __restrict__ w, int R, int C, uint8_t* __restrict__ q, float* __restrict__ s,
                       bool pow2) {
  __shared__ float s_red[8];
  const int rb_n = R / 128, cb_n = C / 128;
  const int64_t blk = blockIdx.x;
  const int64_t mat = blk / ((int64_t)rb_n * cb_n);
  const int rb = (int)((blk / cb_n) % rb_n), cb = (int)(blk % cb_n);
  const T* base = w + mat * (int64_t)R * C + (int64_t)rb * 128 * C + cb * 128;
  uint8_t* qb = q + mat * (int64_t)R * C + (int64_t)rb * 128 * C + cb * 128;
  // thread t covers column t % 128 of rows (t / 128) + 2 * i
  const int col = threadIdx.x & 127, r0 = threadIdx.x >> 7;
  float amax = 0.f;
  for (int r = r0; r < 128; r += 2) amax = fmaxf(amax, fabsf(load_f(base + (int64_t)r * C + col)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float a = threadIdx.x < 8 ? s_red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
    if (threadIdx.x == 0) s_red[0] = a;
  }
  __syncthreads();
  const float sc = fp8_block_scale(s_red[0], pow2);
  for (int r = r0; r < 128; r += 2) qb[(int64_t)r * C + col] = to_e4m3(load_f(base + (int64_t)r * C + col) / sc);
  if (threadIdx.x == 0) s[blk] = sc;
}

}  // namespace

cudaError_t launch_quantize_rows(int dtype, const void* x, int64_t M, int K, uint8_t* q, int64_t ldq, float* s,
                                 int64_t lds, bool pow2, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)ceil_div(M * (K / 128) * 32, 256);
  if (dtype == MOE_DTYPE_BF16)
    quantize_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), M, K, q, ldq,
                                                                s, lds, pow2);
  else if (dtype == MOE_DTYPE_FP16)
    quantize_rows_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x), M, K, q, ldq, s, lds, pow2);
  else
    quantize_rows_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), M, K, q, ldq, s, lds, pow2);
  return cudaGetLastError();
}

}  // namespace moe

extern "C" int moe_quantize_rows_fp8(int dtype, const void* x, int64_t num_rows, int cols, void* q, float* scales,
                                     int scale_fmt, void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16 && dtype != MOE_DTYPE_FP32) return MOE_ERR_UNSUPPORTED;
  if (num_rows < 0 || cols <= 0 || !scale_fmt_ok(scale_fmt)) return MOE_ERR_INVALID_ARG;
  if (cols % 128 != 0) return MOE_ERR_BAD_SHAPE;
  if (num_rows == 0) return MOE_OK;
  if (!x || !q || !scales || (reinterpret_cast<uintptr_t>(q) & 3u)) return MOE_ERR_INVALID_ARG;
  const cudaError_t e = launch_quantize_rows(dtype, x, num_rows, cols, static_cast<uint8_t*>(q), cols, scales,
                                            cols / 128, scale_fmt == MOE_FP8_SCALE_UE8M0,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int64_t moe_fp8_row_bytes(int cols) {
  if (cols <= 0 || cols % 128 != 0) return -1;
  return moe::fp8_row_bytes(cols);
}

extern "C" int moe_quantize_rows_fp8_packed(int dtype, const void* x, int64_t num_rows, int cols, void* rows,
                                            int scale_fmt, void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16 && dtype != MOE_DTYPE_FP32) return MOE_ERR_UNSUPPORTED;
  if (num_rows < 0 || cols <= 0 || !scale_fmt_ok(scale_fmt)) return MOE_ERR_INVALID_ARG;
  if (cols % 128 != 0) return MOE_ERR_BAD_SHAPE;
  if (num_rows == 0) return MOE_OK;
  if (!x || !rows || (reinterpret_cast<uintptr_t>(rows) & 15u)) return MOE_ERR_INVALID_ARG;
  const int64_t rb = fp8_row_bytes(cols);
  uint8_t* r = static_cast<uint8_t*>(rows);
  const cudaError_t e = launch_quantize_rows(dtype, x, num_rows, cols, r, rb, reinterpret_cast<float*>(r + cols),
                                            rb / 4, scale_fmt == MOE_FP8_SCALE_UE8M0,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_quantize_blocks_fp8(int dtype, const void* w, int64_t batch, int rows, int cols, void* q,
                                       float* scales, int scale_fmt, void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16 && dtype != MOE_DTYPE_FP32) return MOE_ERR_UNSUPPORTED;
  if (batch < 0 || rows <= 0 || cols <= 0 || !scale_fmt_ok(scale_fmt)) return MOE_ERR_INVALID_ARG;
  if (rows % 128 != 0 || cols % 128 != 0) return MOE_ERR_BAD_SHAPE;
  if (batch == 0) return MOE_OK;
  if (!w || !q || !scales) return MOE_ERR_INVALID_ARG;
  const int64_t blocks = batch * (rows / 128) * (int64_t)(cols / 128);
  if (blocks > INT32_MAX) return MOE_ERR_BAD_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* qq = static_cast<uint8_t*>(q);
  const bool pow2 = scale_fmt == MOE_FP8_SCALE_UE8M0;
  if (dtype == MOE_DTYPE_BF16)
    quantize_blocks_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), rows,
                                                                           cols, qq, scales, pow2);
  else if (dtype == MOE_DTYPE_FP16)
    quantize_blocks_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __half*>(w), rows, cols, qq,
                                                                    scales, pow2);
  else
    quantize_blocks_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(w), rows, cols, qq,
                                                                   scales, pow2);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

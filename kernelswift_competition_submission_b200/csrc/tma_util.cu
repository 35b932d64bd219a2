// Host-side TMA descriptor encoding (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library needs no link to libcuda).
#include "common.cuh"
#include "moe_internal.h"

#include <mutex>

namespace moe {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

// K-major operand map: innermost box of 64 16-bit elements (128 bytes) with the
// 128-byte swizzle, `box_rows` rows, out-of-bounds elements read as zero.
bool make_kmajor_map(CUtensorMap* m, int dtype, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[3], gstr[2];
  cuuint32_t box[3] = {64, box_rows, 1}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  const CUtensorMapDataType dt =
      dtype == MOE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(m, dt, rank, const_cast<void*>(base), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// e4m3 (byte) operand map: innermost box of 128 bytes (one 128-wide K block) with
// the 128-byte swizzle the tcgen05 descriptors expect; out-of-bounds bytes read as zero.
bool make_fp8_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                  uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[3], gstr[2];
  cuuint32_t box[3] = {128, box_rows, 1}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), gdim, gstr, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 table map, no swizzle: innermost box of `box_rows` elements, one row of the outer dimension.
bool make_f32_rows_map(CUtensorMap* m, const float* base, const uint64_t* dims, const uint64_t* strides_bytes,
                       uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {dims[0], dims[1]}, gstr[1] = {strides_bytes[0]};
  cuuint32_t box[2] = {box_rows, 1}, estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim, gstr, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace moe

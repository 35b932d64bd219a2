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

// Encoded maps, keyed by everything that goes into the encoding (the device's address,
// shape, strides, box, element type, swizzle and the current device). A map encodes only
// addresses and sizes, so a hit is valid whatever happened to the memory in between;
// repeated launches on the same buffers (weights, workspaces) skip the encode call.
struct MapKey {
  int device, kind, dtype, rank;
  const void* base;
  uint64_t dims[3], strides[2];
  uint32_t box_rows;
  bool operator==(const MapKey& o) const {
    return device == o.device && kind == o.kind && dtype == o.dtype && rank == o.rank && base == o.base &&
           dims[0] == o.dims[0] && dims[1] == o.dims[1] && dims[2] == o.dims[2] && strides[0] == o.strides[0] &&
           strides[1] == o.strides[1] && box_rows == o.box_rows;
  }
};

constexpr int kMapCacheSize = 64;
struct MapCache {
  MapKey key[kMapCacheSize];
  CUtensorMap map[kMapCacheSize];
  uint64_t stamp[kMapCacheSize] = {};
  uint64_t clock = 0;
  std::mutex mu;
};
MapCache g_maps;

MapKey map_key(int kind, int dtype, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
               uint32_t box_rows) {
  MapKey k{};
  if (cudaGetDevice(&k.device) != cudaSuccess) k.device = -1;
  k.kind = kind;
  k.dtype = dtype;
  k.rank = rank;
  k.base = base;
  for (int i = 0; i < rank && i < 3; ++i) k.dims[i] = dims[i];
  for (int i = 0; i < rank - 1 && i < 2; ++i) k.strides[i] = strides[i];
  k.box_rows = box_rows;
  return k;
}

bool cache_lookup(const MapKey& k, CUtensorMap* m) {
  std::lock_guard<std::mutex> lock(g_maps.mu);
  for (int i = 0; i < kMapCacheSize; ++i) {
    if (g_maps.stamp[i] && g_maps.key[i] == k) {
      *m = g_maps.map[i];
      g_maps.stamp[i] = ++g_maps.clock;
      return true;
    }
  }
  return false;
}

void cache_store(const MapKey& k, const CUtensorMap& m) {
  std::lock_guard<std::mutex> lock(g_maps.mu);
  int victim = 0;
  for (int i = 1; i < kMapCacheSize; ++i)
    if (g_maps.stamp[i] < g_maps.stamp[victim]) victim = i;  // empty slots (stamp 0) first, then least recent
  g_maps.key[victim] = k;
  g_maps.map[victim] = m;
  g_maps.stamp[victim] = ++g_maps.clock;
}

enum { kMapKMajor16 = 0, kMapFp8 = 1, kMapF32Rows = 2 };

}  // namespace

// K-major operand map: innermost box of 64 16-bit elements (128 bytes) with the
// 128-byte swizzle, `box_rows` rows, out-of-bounds elements read as zero.
bool make_kmajor_map(CUtensorMap* m, int dtype, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, uint32_t box_rows) {
  const MapKey key = map_key(kMapKMajor16, dtype, base, rank, dims, strides_bytes, box_rows);
  if (cache_lookup(key, m)) return true;
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[3], gstr[2];
  cuuint32_t box[3] = {64, box_rows, 1}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  const CUtensorMapDataType dt =
      dtype == MOE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (enc(m, dt, rank, const_cast<void*>(base), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return false;
  cache_store(key, *m);
  return true;
}

// e4m3 (byte) operand map: innermost box of 128 bytes (one 128-wide K block) with
// the 128-byte swizzle the tcgen05 descriptors expect; out-of-bounds bytes read as zero.
bool make_fp8_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                  uint32_t box_rows) {
  const MapKey key = map_key(kMapFp8, 0, base, rank, dims, strides_bytes, box_rows);
  if (cache_lookup(key, m)) return true;
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[3], gstr[2];
  cuuint32_t box[3] = {128, box_rows, 1}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  if (enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), gdim, gstr, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cache_store(key, *m);
  return true;
}

// fp32 table map, no swizzle: innermost box of `box_rows` elements, one row of the outer dimension.
bool make_f32_rows_map(CUtensorMap* m, const float* base, const uint64_t* dims, const uint64_t* strides_bytes,
                       uint32_t box_rows) {
  const MapKey key = map_key(kMapF32Rows, 0, base, 2, dims, strides_bytes, box_rows);
  if (cache_lookup(key, m)) return true;
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {dims[0], dims[1]}, gstr[1] = {strides_bytes[0]};
  cuuint32_t box[2] = {box_rows, 1}, estr[2] = {1, 1};
  if (enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim, gstr, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cache_store(key, *m);
  return true;
}

// Raises a kernel's dynamic shared-memory limit once per (function, device) and size.
cudaError_t ensure_smem_limit(const void* func, int bytes) {
  struct Entry {
    const void* func;
    int device, bytes;
  };
  static Entry entries[256];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (entries[i].func == func && entries[i].device == dev && entries[i].bytes >= bytes) return cudaSuccess;
  err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess) return err;
  for (int i = 0; i < n; ++i)
    if (entries[i].func == func && entries[i].device == dev) {
      entries[i].bytes = bytes;
      return cudaSuccess;
    }
  if (n < 256) entries[n++] = Entry{func, dev, bytes};
  return cudaSuccess;
}

}  // namespace moe

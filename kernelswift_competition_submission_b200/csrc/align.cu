// Align stage: counting sort of the (token, slot) pairs by expert, each
// expert's segment padded to a multiple of block_m rows, plus (fused path) the
// gather of each pair's token row into expert-sorted order.
//
// Replaces the per-expert boolean masks and host syncs of
// fused_moe/v0/fused_moe.py:143-159 (`mask = flat_ids == e; if not mask.any()`)
// with two launches and no host round trip:
//   1. align_count_kernel: per-CTA shared-memory histograms added into global
//      counts; the last CTA to finish scans them into block_start (m-blocks per
//      expert), writes the total and marks padding rows with -1.
//   2. align_scatter_kernel: each CTA re-histograms its chunk, reserves one
//      range per expert with a single global atomic, writes its pair ids and,
//      when asked, copies the token rows (warp per row, 16-byte vectors).
// Pair order inside an expert segment is unspecified; every output row of the
// GEMMs depends only on its own pair, so results do not depend on it.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>
#include <mutex>

namespace moe {
namespace {

constexpr int kAlignThreads = 512;
constexpr int kScatterChunk = 1024;  // pairs per scatter CTA

__global__ void __launch_bounds__(kAlignThreads)
align_count_kernel(const int32_t* __restrict__ ids, int64_t P, int E, int bm, AlignMeta m,
                   int32_t* __restrict__ sorted_pairs, int64_t cap) {
  extern __shared__ int s_hist[];  // [E]
  __shared__ int s_last;
  for (int i = threadIdx.x; i < E; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < P; p += stride) {
    const int e = __ldg(ids + p);
    if (e >= 0 && e < E) atomicAdd(&s_hist[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (s_hist[i]) atomicAdd(&m.counts[i], s_hist[i]);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(m.done, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last CTA: exclusive scan of ceil(count / bm) over experts (E <= 1024).
  int* s_blk = s_hist;  // reuse
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    const int c = __ldcg(&m.counts[i]);
    s_blk[i] = (c + bm - 1) / bm;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // one warp scans: each lane owns a contiguous run of ceil(E/32) experts
    const int lane = threadIdx.x;
    const int per = (E + 31) / 32;
    const int b = lane * per;
    int local = 0;
    for (int i = 0; i < per; ++i)
      if (b + i < E) local += s_blk[b + i];
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int run = incl - local;
    for (int i = 0; i < per; ++i) {
      if (b + i < E) {
        const int nb = s_blk[b + i];
        m.block_start[b + i] = run;
        s_blk[b + i] = run;  // now the start
        run += nb;
      }
    }
    if (lane == 31) m.block_start[E] = incl;
  }
  __syncthreads();
  // padding rows of each expert's last m-block -> -1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int e = warp; e < E; e += nwarps) {
    const int c = __ldcg(&m.counts[e]);
    const int64_t r0 = (int64_t)s_blk[e] * bm + c;
    const int64_t r1 = (int64_t)(s_blk[e] + (c + bm - 1) / bm) * bm;
    for (int64_t r = r0 + lane; r < r1 && r < cap; r += 32) sorted_pairs[r] = -1;
  }
}

__global__ void __launch_bounds__(kAlignThreads)
align_scatter_kernel(const int32_t* __restrict__ ids, int64_t P, int topk, int E, int bm, AlignMeta m,
                     int32_t* __restrict__ sorted_pairs, const uint4* __restrict__ x_src,
                     uint4* __restrict__ x_sorted, int64_t row_vecs) {
  extern __shared__ int s_dyn[];
  int* s_hist = s_dyn;          // [E]
  int* s_base = s_dyn + E;      // [E]
  __shared__ int s_e[kScatterChunk];
  __shared__ int s_pos[kScatterChunk];
  const int64_t c0 = (int64_t)blockIdx.x * kScatterChunk;
  const int n = (int)((P - c0) < kScatterChunk ? (P - c0) : kScatterChunk);
  for (int i = threadIdx.x; i < E; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = __ldg(ids + c0 + i);
    const bool ok = e >= 0 && e < E;
    s_e[i] = ok ? e : -1;
    s_pos[i] = ok ? atomicAdd(&s_hist[e], 1) : -1;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int h = s_hist[e];
    s_base[e] = h ? __ldg(&m.block_start[e]) * bm + atomicAdd(&m.cursor[e], h) : 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = s_e[i];
    if (e >= 0) {
      const int r = s_base[e] + s_pos[i];
      s_pos[i] = r;
      sorted_pairs[r] = (int32_t)(c0 + i);
    }
  }
  if (x_src == nullptr) return;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int i = warp; i < n; i += nwarps) {
    if (s_e[i] < 0) continue;
    const int64_t tok = (c0 + i) / topk;
    const uint4* src = x_src + tok * row_vecs;
    uint4* dst = x_sorted + (int64_t)s_pos[i] * row_vecs;
    int64_t v = lane;
    for (; v + 96 < row_vecs; v += 128) {
      const uint4 a = __ldg(src + v), b = __ldg(src + v + 32), c = __ldg(src + v + 64), d = __ldg(src + v + 96);
      dst[v] = a; dst[v + 32] = b; dst[v + 64] = c; dst[v + 96] = d;
    }
    for (; v < row_vecs; v += 32) dst[v] = __ldg(src + v);
  }
}

}  // namespace

cudaError_t launch_align(const int32_t* topk_ids, int64_t P, int topk, int E, int bm, AlignMeta meta,
                         bool meta_contiguous, int32_t* sorted_pairs, int64_t cap, const void* x_src, void* x_sorted,
                         int64_t row_bytes, cudaStream_t st, bool zero_meta) {
  cudaError_t err = cudaSuccess;
  if (zero_meta && meta_contiguous) {
    err = cudaMemsetAsync(meta.counts, 0, sizeof(int32_t) * (2 * (size_t)E + 1), st);
  } else if (zero_meta) {
    err = cudaMemsetAsync(meta.counts, 0, sizeof(int32_t) * E, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(meta.cursor, 0, sizeof(int32_t) * E, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(meta.done, 0, sizeof(int32_t), st);
  }
  if (err != cudaSuccess) return err;
  const int count_blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(P, kAlignThreads * 8), 2 * num_sms()));
  align_count_kernel<<<count_blocks, kAlignThreads, sizeof(int) * E, st>>>(topk_ids, P, E, bm, meta, sorted_pairs, cap);
  err = cudaGetLastError();
  if (err != cudaSuccess || P == 0) return err;
  const int scatter_blocks = (int)ceil_div(P, kScatterChunk);
  align_scatter_kernel<<<scatter_blocks, kAlignThreads, sizeof(int) * 2 * E, st>>>(
      topk_ids, P, topk, E, bm, meta, sorted_pairs, static_cast<const uint4*>(x_src), static_cast<uint4*>(x_sorted),
      row_bytes / 16);
  return cudaGetLastError();
}

int num_sms() {
  static int cache[64];  // per device, 0 = not read yet
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return n;
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

}  // namespace moe

extern "C" int64_t moe_align_capacity(int64_t num_pairs, int num_experts, int block_m) {
  if (num_pairs < 0 || num_experts <= 0 || block_m <= 0) return -1;
  // every expert's segment rounds up to a whole m-block
  const int64_t cap = num_pairs + (int64_t)num_experts * (block_m - 1);
  return moe::ceil_div(cap, block_m) * block_m;
}

extern "C" int moe_align(const int32_t* topk_ids, int64_t num_pairs, int num_experts, int block_m, int32_t* counts,
                         int32_t* block_start, int32_t* sorted_pairs, int64_t sorted_capacity, int32_t* scratch,
                         void* stream) {
  if (num_pairs < 0 || num_experts <= 0 || num_experts > 1024 || block_m <= 0 || block_m > 4096)
    return MOE_ERR_INVALID_ARG;
  if (!counts || !block_start || !scratch || (num_pairs > 0 && (!topk_ids || !sorted_pairs)))
    return MOE_ERR_INVALID_ARG;
  if (num_pairs > INT32_MAX) return MOE_ERR_BAD_SHAPE;
  if (sorted_capacity < moe_align_capacity(num_pairs, num_experts, block_m)) return MOE_ERR_WORKSPACE;
  moe::AlignMeta m{counts, scratch, block_start, scratch + num_experts};
  const cudaError_t err = moe::launch_align(topk_ids, num_pairs, 1, num_experts, block_m, m, false, sorted_pairs,
                                            sorted_capacity, nullptr, nullptr, 0, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// moe_align_noalloc: the align stage for callers that cannot hand this library
// any device memory of their own.
//
// Its only scratch (one cursor per expert plus the CTA completion counter) is
// the fixed array below, sized for MOE_NOALLOC_MAX_EXPERTS experts (4100 bytes).
// Every GPU that loads this library holds it until the process exits. Host code
// must not pass `g_noalloc_align_scratch` itself to a kernel (on the host that
// name is only a stand-in); the device address is looked up once per device
// with cudaGetSymbolAddress, on the first call made while that device is
// current, and cached.
namespace {

static __device__ __align__(256) int32_t g_noalloc_align_scratch[MOE_NOALLOC_MAX_EXPERTS + 1];

constexpr int kNoAllocMaxDevices = 64;
int32_t* g_noalloc_scratch_ptr[kNoAllocMaxDevices];
std::mutex g_noalloc_mutex;

int noalloc_scratch(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return MOE_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_align_scratch) != cudaSuccess || p == nullptr) return MOE_ERR_CUDA;
    g_noalloc_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_noalloc_scratch_ptr[dev];
  return MOE_OK;
}

}  // namespace

extern "C" int moe_align_noalloc(const int32_t* topk_ids, int64_t num_pairs, int num_experts, int block_m,
                                 int32_t* counts, int32_t* block_start, int32_t* sorted_pairs,
                                 int64_t sorted_capacity, void* stream) {
  if (num_experts > MOE_NOALLOC_MAX_EXPERTS) return MOE_ERR_SCRATCH_LIMIT;
  if (num_pairs < 0 || num_experts <= 0 || block_m <= 0 || block_m > 4096) return MOE_ERR_INVALID_ARG;
  if (!counts || !block_start || (num_pairs > 0 && (!topk_ids || !sorted_pairs))) return MOE_ERR_INVALID_ARG;
  if (num_pairs > INT32_MAX) return MOE_ERR_BAD_SHAPE;
  if (sorted_capacity < moe_align_capacity(num_pairs, num_experts, block_m)) return MOE_ERR_WORKSPACE;
  int32_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != MOE_OK) return rc;
  // cursor = scratch[0, E), done = scratch[E]; launch_align zeroes both (and counts)
  // on `stream` before its kernels run, so the previous call's contents never leak in.
  moe::AlignMeta m{counts, scratch, block_start, scratch + num_experts};
  const cudaError_t err = moe::launch_align(topk_ids, num_pairs, 1, num_experts, block_m, m, false, sorted_pairs,
                                            sorted_capacity, nullptr, nullptr, 0, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

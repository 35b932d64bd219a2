// Expert-parallel dispatch / combine over NVLink peer memory, for decode-sized
// batches where an all-to-all's fixed latency and the host round trip of its split
// sizes dominate. Every rank owns one arena (cudaMalloc, shared with the other ranks
// through CUDA IPC handles):
//
//   ctrl    ready[world] | disp[world] | back[world] | counts[world]   (u32 / int32)
//   recv_x  [world][cap][K]       token rows sent to this rank, region = source rank (bf16 /
//                                 fp16, or packed e4m3 rows at their own smaller pitch)
//   recv_id [world][cap][k]       expert ids in this rank's numbering (-1: not this rank's)
//   recv_w  [world][cap][k]       the token's top-k weights
//   back_x  [world][cap][K]       partial rows returned to this rank, region = expert rank
//
// One step s (seq numbers only grow; every flag is written with release and read with
// acquire at system scope; every wait is bounded and records MOE_ERR_TIMEOUT):
//   1. signal ready[me] = s in every rank: this rank's arena is free again (its previous
//      step finished in stream order).
//   2. dispatch: wait until every rank is ready for s; one warp per token writes the
//      token's row, ids and weights straight into each destination rank's region `me`
//      (NVLink stores); the last CTA clears the id rows this source used last step but
//      not now, publishes counts[me] and then disp[me] = s in each destination.
//   3. wait disp[*] = s; the local expert path runs over all world * cap rows (unused
//      rows carry id -1 and are skipped).
//   4. combine_back: each returned partial row goes to back_x region `me` of its source
//      rank at the row the source wrote it; the last CTA sets back[me] = s there.
//   5. wait back[*] = s; the source sums its token's returned rows (moe_ep_combine).
// No NCCL and no host synchronisation on the data path; no multicast objects.
//
// Failure: a wait that gives up records MOE_ERR_TIMEOUT in the caller's status word.
// Every kernel here reads that word first and, once it is set, does nothing: no waits,
// no stores into other ranks' arenas, no flags. A rank that timed out therefore goes
// quiet, the ranks waiting on it time out in turn, and moe_p2p_reduce writes NaN rows
// instead of summing a step whose rows never arrived. The host learns of it from the
// status word and rebuilds the arenas (collectively) before the next step.
#include "common.cuh"
#include "moe_internal.h"

#include <algorithm>

namespace moe {
namespace {

constexpr int kP2PThreads = 256;
constexpr int kP2PMaxWorld = 64;

struct P2PLayout {
  int64_t ready, disp, back, counts, recv_x, recv_id, recv_w, back_x, total;
};

inline int64_t up256(int64_t v) { return (v + 255) / 256 * 256; }

P2PLayout p2p_layout(int world, int64_t cap, int K, int topk) {
  P2PLayout l;
  int64_t o = 0;
  l.ready = o;   o += 4 * world;
  l.disp = o;    o += 4 * world;
  l.back = o;    o += 4 * world;
  l.counts = o;  o = up256(o + 4 * world);
  l.recv_x = o;  o = up256(o + (int64_t)world * cap * K * 2);
  l.recv_id = o; o = up256(o + (int64_t)world * cap * topk * 4);
  l.recv_w = o;  o = up256(o + (int64_t)world * cap * topk * 4);
  l.back_x = o;  o = up256(o + (int64_t)world * cap * K * 2);
  l.total = o;
  return l;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// seq numbers wrap modulo 2^32: "reached" means no more than 2^31 behind
__device__ __forceinline__ bool reached(uint32_t v, uint32_t seq) { return (int32_t)(v - seq) >= 0; }

// Set once a wait of this rank gave up (or any earlier failure was recorded).
__device__ __forceinline__ bool failed(const int* status) {
  return status != nullptr && *reinterpret_cast<const volatile int*>(status) != 0;
}

// Bounded wait (thread-level) until flags[0..world) have all reached seq.
__device__ bool wait_flags(const uint32_t* flags, int world, uint32_t seq, int* status) {
  const uint64_t t0 = globaltimer_ns();
  for (int d = 0; d < world; ++d) {
    while (!reached(ld_acquire_sys(flags + d), seq)) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(status, MOE_ERR_TIMEOUT);
        return false;
      }
      __nanosleep(128);
    }
  }
  return true;
}

__global__ void p2p_signal_kernel(const int64_t* __restrict__ peer_base, int world, int me, int64_t flag_off,
                                  uint32_t seq, const int* status) {
  const int d = threadIdx.x;
  if (d < world && !failed(status)) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(peer_base[d] + flag_off) + me, seq);
  }
}

__global__ void p2p_wait_kernel(const uint32_t* flags, int world, uint32_t seq, int* status) {
  if (threadIdx.x == 0 && !failed(status)) wait_flags(flags, world, seq, status);
}

// scratch: [world] rows claimed this step | [world] rows used last step | [1] CTAs done
__global__ void __launch_bounds__(kP2PThreads)
p2p_dispatch_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ ids, const float* __restrict__ w,
                    int64_t M, int64_t row_vecs, int topk, int epr, int world, int me, int64_t cap,
                    const int64_t* __restrict__ peer_base, P2PLayout lay, uint32_t seq, int32_t* scratch,
                    int32_t* __restrict__ tok_rows, const uint32_t* own_ready, int* status) {
  __shared__ int s_go, s_last;
  int32_t* claimed = scratch;
  int32_t* used = scratch + world;
  int32_t* done = scratch + 2 * world;
  if (threadIdx.x == 0) s_go = (!failed(status) && wait_flags(own_ready, world, seq, status)) ? 1 : 0;
  __syncthreads();
  if (!s_go) return;  // failed: touch no arena and raise no flag (the step's output becomes NaN)
  const int lane = threadIdx.x & 31;
  {
    for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < M;
         t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
      uint64_t mask = 0;
      for (int j = 0; j < topk; ++j) {
        const int e = __ldg(ids + t * topk + j);
        if (e >= 0 && e < epr * world) mask |= 1ull << (e / epr);
      }
      const int my_e = lane < topk ? __ldg(ids + t * topk + lane) : -1;
      const float my_w = lane < topk ? __ldg(w + t * topk + lane) : 0.f;
      // destinations in the order me, me + 1, ...: the ranks do not all start on rank 0
      for (int i = 0; i < world; ++i) {
        const int d = me + i < world ? me + i : me + i - world;
        int r = -1;
        if ((mask >> d) & 1ull) {
          if (lane == 0) r = atomicAdd(claimed + d, 1);
          r = __shfl_sync(0xffffffffu, r, 0);
          const int64_t row = (int64_t)me * cap + r;  // region `me` of rank d
          char* base = reinterpret_cast<char*>(peer_base[d]);
          uint4* dst = reinterpret_cast<uint4*>(base + lay.recv_x) + row * row_vecs;
          const uint4* src = x + t * row_vecs;
          // four 16-byte loads in flight per lane before their stores
          int64_t v = lane;
          for (; v + 96 < row_vecs; v += 128) {
            const uint4 a0 = __ldg(src + v), a1 = __ldg(src + v + 32), a2 = __ldg(src + v + 64),
                        a3 = __ldg(src + v + 96);
            dst[v] = a0;
            dst[v + 32] = a1;
            dst[v + 64] = a2;
            dst[v + 96] = a3;
          }
          for (; v < row_vecs; v += 32) dst[v] = __ldg(src + v);
          if (lane < topk) {
            const bool own = my_e >= 0 && my_e < epr * world && my_e / epr == d;
            reinterpret_cast<int32_t*>(base + lay.recv_id)[row * topk + lane] = own ? my_e - d * epr : -1;
            reinterpret_cast<float*>(base + lay.recv_w)[row * topk + lane] = my_w;
          }
        }
        if (lane == 0) tok_rows[t * world + d] = r < 0 ? -1 : (int32_t)((int64_t)d * cap + r);
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(done, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // last CTA: clear the id rows used last step and not now, publish counts, then the flag
  for (int d = 0; d < world; ++d) {
    const int n = __ldcg(claimed + d);
    const int p = used[d];
    char* base = reinterpret_cast<char*>(peer_base[d]);
    int32_t* rid = reinterpret_cast<int32_t*>(base + lay.recv_id);
    for (int64_t i = (int64_t)n * topk + threadIdx.x; i < (int64_t)p * topk; i += blockDim.x)
      rid[(int64_t)me * cap * topk + i] = -1;
  }
  __threadfence_system();  // every thread's clears ordered before the flags below
  __syncthreads();
  if (threadIdx.x < world) {
    const int d = threadIdx.x;
    const int n = __ldcg(claimed + d);
    char* base = reinterpret_cast<char*>(peer_base[d]);
    reinterpret_cast<volatile int32_t*>(base + lay.counts)[me] = n;
    used[d] = n;
    claimed[d] = 0;
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(base + lay.disp) + me, seq);
  }
  if (threadIdx.x == 0) *done = 0;
}

// partial [world * cap, K]: row src * cap + r is the expert output of the r-th row that
// rank src sent here; it goes to rank src's back_x region `me`, row r.
__global__ void __launch_bounds__(kP2PThreads)
p2p_combine_back_kernel(const uint4* __restrict__ partial, int K, int world, int me, int64_t cap,
                        const int64_t* __restrict__ peer_base, P2PLayout lay, const int32_t* own_counts,
                        uint32_t seq, int32_t* done, const int* status) {
  __shared__ int s_last;
  if (failed(status)) return;
  const int lane = threadIdx.x & 31;
  const int64_t row_vecs = (int64_t)K * 2 / 16;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < (int64_t)world * cap;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int src = (int)(row / cap);
    const int64_t r = row - (int64_t)src * cap;
    if (r >= __ldcg(own_counts + src)) continue;
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(peer_base[src]) + lay.back_x) +
                 ((int64_t)me * cap + r) * row_vecs;
    const uint4* s = partial + row * row_vecs;
    for (int64_t v = lane; v < row_vecs; v += 32) dst[v] = __ldg(s + v);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(done, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  if (threadIdx.x < world)
    st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(peer_base[threadIdx.x]) + lay.back) + me,
                   seq);
  if (threadIdx.x == 0) *done = 0;
}

// The expert path's top-k combine fused with the return trip, one warp per received row:
// for row t (region src = t / cap, row r = t % cap, r < counts[src]) the lanes read the
// row's k ids and weights once, then the weighted sum of its valid slot rows of y_slots
// (slots in order, fmaf per slot: the bits of combine_kernel) is stored 16 bytes per lane
// straight into rank src's back_x region `me`, row r, four vectors per lane at a time
// with the loads of a slot issued before its FMAs. The grid strides over the rows; each
// CTA issues its system-scope fence once; the last CTA raises back[me] in every rank.
template <typename T>
__global__ void __launch_bounds__(kP2PThreads)
p2p_combine_experts_back_kernel(const uint4* __restrict__ y, const float* __restrict__ w,
                                const int32_t* __restrict__ ids, int E, int topk, int vpr, int world, int me,
                                int64_t cap, const int64_t* __restrict__ peer_base, P2PLayout lay,
                                const int32_t* own_counts, uint32_t seq, int32_t* done, const int* status) {
  __shared__ int s_last;
  __shared__ int s_cnt[kP2PMaxWorld];
  if (failed(status)) return;
  for (int i = threadIdx.x; i < world; i += blockDim.x) s_cnt[i] = __ldcg(own_counts + i);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)world * cap;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < rows; t += nwarps) {
    const int src = (int)(t / cap);
    const int64_t r = t - (int64_t)src * cap;
    if (r >= s_cnt[src]) continue;  // warp-uniform
    const int e = lane < topk ? __ldg(ids + t * topk + lane) : -1;
    const float my_w = lane < topk ? __ldg(w + t * topk + lane) : 0.f;
    const uint32_t valid = __ballot_sync(0xffffffffu, e >= 0 && e < E);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(peer_base[src]) + lay.back_x) +
                 ((int64_t)me * cap + r) * vpr;
    const uint4* yr = y + t * topk * (int64_t)vpr;
    for (int v0 = lane; v0 < vpr; v0 += 128) {
      float acc[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
      for (uint32_t m = valid; m; m &= m - 1) {  // slots in order
        const int j = __ffs(m) - 1;
        const float wj = __shfl_sync(0xffffffffu, my_w, j);
        const uint4* ys = yr + (int64_t)j * vpr;
        uint4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) q[u] = v0 + 32 * u < vpr ? __ldg(ys + v0 + 32 * u) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t h[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = ElemTraits<T>::unpack2(h[i]);
            acc[u][2 * i] = fmaf(wj, f.x, acc[u][2 * i]);
            acc[u][2 * i + 1] = fmaf(wj, f.y, acc[u][2 * i + 1]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (v0 + 32 * u < vpr) {
          uint4 o;
          o.x = ElemTraits<T>::pack2(acc[u][0], acc[u][1]);
          o.y = ElemTraits<T>::pack2(acc[u][2], acc[u][3]);
          o.z = ElemTraits<T>::pack2(acc[u][4], acc[u][5]);
          o.w = ElemTraits<T>::pack2(acc[u][6], acc[u][7]);
          dst[v0 + 32 * u] = o;
        }
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(done, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  if (threadIdx.x < world)
    st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(peer_base[threadIdx.x]) + lay.back) + me,
                   seq);
  if (threadIdx.x == 0) *done = 0;
}

inline bool p2p_ok(int world, int me, int64_t cap, int K, int topk) {
  return world > 0 && world <= kP2PMaxWorld && me >= 0 && me < world && cap > 0 && K > 0 && K % 8 == 0 &&
         topk > 0 && topk <= 32;
}

}  // namespace
}  // namespace moe

extern "C" int64_t moe_p2p_arena_bytes(int world, int64_t cap, int hidden_size, int topk) {
  if (!moe::p2p_ok(world, 0, cap, hidden_size, topk)) return -1;
  return moe::p2p_layout(world, cap, hidden_size, topk).total;
}

extern "C" int moe_p2p_arena_offsets(int world, int64_t cap, int hidden_size, int topk, int64_t* offsets) {
  if (!moe::p2p_ok(world, 0, cap, hidden_size, topk) || !offsets) return MOE_ERR_INVALID_ARG;
  const moe::P2PLayout l = moe::p2p_layout(world, cap, hidden_size, topk);
  const int64_t v[9] = {l.ready, l.disp, l.back, l.counts, l.recv_x, l.recv_id, l.recv_w, l.back_x, l.total};
  for (int i = 0; i < 9; ++i) offsets[i] = v[i];
  return MOE_OK;
}

extern "C" int moe_p2p_alloc(int world, int64_t cap, int hidden_size, int topk, void** base, void* ipc_handle) {
  using namespace moe;
  if (!p2p_ok(world, 0, cap, hidden_size, topk) || !base || !ipc_handle) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)l.total) != cudaSuccess) return MOE_ERR_CUDA;
  // flags and counts [0, recv_x) zero; everything after it 0xFF: id rows -1 (no token)
  if (cudaMemset(p, 0, (size_t)l.recv_x) != cudaSuccess ||
      cudaMemset(static_cast<char*>(p) + l.recv_x, 0xFF, (size_t)(l.total - l.recv_x)) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return MOE_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return MOE_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *base = p;
  return MOE_OK;
}

extern "C" int moe_p2p_open(const void* ipc_handle, void** base) {
  if (!ipc_handle || !base) return MOE_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_close(void* base) {
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_free(void* base) { return cudaFree(base) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA; }

extern "C" int moe_p2p_signal(const int64_t* peer_bases, int world, int me, int which, int64_t cap, int hidden_size,
                              int topk, uint32_t seq, int* status, void* stream) {
  using namespace moe;
  if (!p2p_ok(world, me, cap, hidden_size, topk) || !peer_bases || which < 0 || which > 2) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  const int64_t off = which == 0 ? l.ready : which == 1 ? l.disp : l.back;
  p2p_signal_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(peer_bases, world, me, off, seq, status);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_wait(const void* own_base, int world, int which, int64_t cap, int hidden_size, int topk,
                            uint32_t seq, int* status, void* stream) {
  using namespace moe;
  if (!p2p_ok(world, 0, cap, hidden_size, topk) || !own_base || which < 0 || which > 2) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  const int64_t off = which == 0 ? l.ready : which == 1 ? l.disp : l.back;
  p2p_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(static_cast<const char*>(own_base) + off), world, seq, status);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_dispatch(int dtype, const void* hidden_states, const int32_t* topk_ids,
                                const float* topk_weights, int64_t num_tokens, int hidden_size, int topk,
                                int experts_per_rank, int world, int me, int64_t cap, const int64_t* peer_bases,
                                const void* own_base, uint32_t seq, int32_t* scratch, int32_t* tok_rows, int* status,
                                void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16 && dtype != MOE_DTYPE_E4M3_ROW) return MOE_ERR_UNSUPPORTED;
  if (!p2p_ok(world, me, cap, hidden_size, topk) || experts_per_rank <= 0 || num_tokens < 0 || num_tokens > cap)
    return MOE_ERR_INVALID_ARG;
  if (dtype == MOE_DTYPE_E4M3_ROW && hidden_size % 128 != 0) return MOE_ERR_BAD_SHAPE;
  if (!peer_bases || !own_base || !scratch || !tok_rows || (num_tokens > 0 && (!hidden_states || !topk_ids ||
                                                                              !topk_weights)))
    return MOE_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(hidden_states) & 15u) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(num_tokens * 32, kP2PThreads), 2 * num_sms()));
  const uint32_t* own_ready = reinterpret_cast<const uint32_t*>(static_cast<const char*>(own_base) + l.ready);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 16-byte vectors per row; a packed e4m3 row (K + K / 32 bytes, rounded up) fits the
  // K * 2 bytes a recv_x row holds, and is stored at that smaller pitch
  const int64_t row_vecs = (dtype == MOE_DTYPE_E4M3_ROW ? fp8_row_bytes(hidden_size) : (int64_t)hidden_size * 2) / 16;
  p2p_dispatch_kernel<<<blocks, kP2PThreads, 0, st>>>(
      static_cast<const uint4*>(hidden_states), topk_ids, topk_weights, num_tokens, row_vecs, topk, experts_per_rank,
      world, me, cap, peer_bases, l, seq, scratch, tok_rows, own_ready, status);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_combine_back(int dtype, const void* partial, int hidden_size, int topk, int world, int me,
                                    int64_t cap, const int64_t* peer_bases, const void* own_base, uint32_t seq,
                                    int32_t* scratch, int* status, void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16) return MOE_ERR_UNSUPPORTED;
  if (!p2p_ok(world, me, cap, hidden_size, topk) || !partial || !peer_bases || !own_base || !scratch)
    return MOE_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(partial) & 15u) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  const int64_t rows = (int64_t)world * cap;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows * 32, kP2PThreads), 2 * num_sms()));
  const int32_t* own_counts = reinterpret_cast<const int32_t*>(static_cast<const char*>(own_base) + l.counts);
  p2p_combine_back_kernel<<<blocks, kP2PThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(partial), hidden_size, world, me, cap, peer_bases, l, own_counts, seq, scratch,
      status);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_copy_recv_ids(const void* own_base, int world, int64_t cap, int hidden_size, int topk,
                                     int32_t* dst, void* stream) {
  using namespace moe;
  if (!p2p_ok(world, 0, cap, hidden_size, topk) || !own_base || !dst) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  return cudaMemcpyAsync(dst, static_cast<const char*>(own_base) + l.recv_id, sizeof(int32_t) * world * cap * topk,
                         cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? MOE_OK
             : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_combine_experts_back(int dtype, const void* workspace, int num_experts, int hidden_size,
                                            int intermediate_size, int topk, int world, int me, int64_t cap,
                                            const int64_t* peer_bases, const void* own_base, uint32_t seq,
                                            int32_t* scratch, int* status, void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16 && dtype != MOE_DTYPE_E4M3_ROW) return MOE_ERR_UNSUPPORTED;
  if (!p2p_ok(world, me, cap, hidden_size, topk) || num_experts <= 0 || intermediate_size <= 0 || !workspace ||
      !peer_bases || !own_base || !scratch)
    return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  const int64_t R = (int64_t)world * cap;
  // the slot rows the expert path left in its workspace (bf16 for the FP8 path)
  const size_t y_off = dtype == MOE_DTYPE_E4M3_ROW
                           ? fp8_yslots_offset(R, num_experts, topk, hidden_size, intermediate_size)
                           : fused_yslots_offset(R, num_experts, topk, hidden_size, intermediate_size);
  const uint4* y = reinterpret_cast<const uint4*>(static_cast<const char*>(workspace) + y_off);
  const char* ob = static_cast<const char*>(own_base);
  const int vpr = hidden_size / 8;
  // one warp per received row; up to 4 CTAs of 8 warps per SM (64 registers)
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(R * 32, kP2PThreads), 4 * num_sms()));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* w = reinterpret_cast<const float*>(ob + l.recv_w);
  const int32_t* ids = reinterpret_cast<const int32_t*>(ob + l.recv_id);
  const int32_t* cnt = reinterpret_cast<const int32_t*>(ob + l.counts);
  if (dtype != MOE_DTYPE_FP16)
    p2p_combine_experts_back_kernel<__nv_bfloat16><<<blocks, kP2PThreads, 0, st>>>(
        y, w, ids, num_experts, topk, vpr, world, me, cap, peer_bases, l, cnt, seq, scratch, status);
  else
    p2p_combine_experts_back_kernel<__half><<<blocks, kP2PThreads, 0, st>>>(
        y, w, ids, num_experts, topk, vpr, world, me, cap, peer_bases, l, cnt, seq, scratch, status);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_p2p_reduce(int dtype, const void* own_base, const int32_t* tok_rows, int64_t num_tokens,
                              int hidden_size, int topk, int world, int64_t cap, void* out, const int* status,
                              void* stream) {
  using namespace moe;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP16) return MOE_ERR_UNSUPPORTED;
  if (!p2p_ok(world, 0, cap, hidden_size, topk) || num_tokens < 0 || num_tokens > cap || !own_base ||
      (num_tokens > 0 && (!tok_rows || !out)))
    return MOE_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(out) & 15u) return MOE_ERR_INVALID_ARG;
  const P2PLayout l = p2p_layout(world, cap, hidden_size, topk);
  return launch_ep_combine(dtype, static_cast<const char*>(own_base) + l.back_x, tok_rows, num_tokens, hidden_size,
                           world, out, status, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? MOE_OK
             : MOE_ERR_CUDA;
}

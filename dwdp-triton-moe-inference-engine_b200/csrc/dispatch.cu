// Dispatcher: stable counting sort of token-major (token, slot) assignments
// into expert-major order, bit-exact with the reference counting scatter
// (DWDP/dispatcher/kernels/reference.py:163-257 with
// DWDP/dispatcher/ops/scatter.py:6-96):
//
//   counts[e]   = #{i : e_i == e}
//   offsets     = exclusive prefix sum of counts (E + 1 entries)
//   dest[i]     = offsets[e_i] + #{j < i : e_j == e_i}        (stable)
//   perm[dest]  = i,  inv[i] = dest,  ids[dest] = e_i,
//   tok[dest]   = i / K,  packed_w[dest] = w_i (bit copy)
//
// Up to three launches, no host synchronisation:
//   1. tile histogram: each CTA of kTile assignments writes int32 counts [E]
//      into the caller's scratch (skipped for a single tile, T * K <= kTile:
//      the scatter CTA counts its own elements)
//   2. scatter: each CTA reduces the tile histograms before it (its exclusive
//      start inside each expert segment) and all of them (global counts ->
//      offsets), ranks its own elements stably with warp match masks plus
//      per-warp counts in shared memory, and writes the index arrays
//   3. row gather: packed_hidden[d] = hidden[tok[d]] with 16-byte vectors,
//      one warp per row (an HBM-bound copy)
#include "common.cuh"

namespace dwdp {

constexpr int kTile = 256;  // assignments per CTA (one per thread)
constexpr int kMaxExperts = 1024;

__global__ void __launch_bounds__(kTile)
dispatch_hist_kernel(const int64_t* __restrict__ idx, int64_t N, int E, int* __restrict__ tile_hist,
                     DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  __shared__ int h[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * kTile + threadIdx.x;
  if (i < N) {
    const int64_t e = idx[i];
    if (e >= 0 && e < E) {
      atomicAdd(&h[e], 1);
    } else {
      record_error(st, DWDP_ERR_DEVICE_BOUNDS, 100, (int)i);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) tile_hist[(int64_t)blockIdx.x * E + e] = h[e];
}

template <typename TWt>
__global__ void __launch_bounds__(kTile)
dispatch_scatter_kernel(const int64_t* __restrict__ idx, const TWt* __restrict__ wts, int64_t N,
                        int K, int E, int ntiles, const int* __restrict__ tile_hist,
                        int64_t* __restrict__ counts, int64_t* __restrict__ offsets,
                        int64_t* __restrict__ perm, int64_t* __restrict__ inv,
                        int64_t* __restrict__ ids, int64_t* __restrict__ tok,
                        TWt* __restrict__ packed_w, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  __shared__ int s_start[kMaxExperts];  // offsets[e] + tiles-before prefix
  __shared__ int s_tot[kMaxExperts];
  __shared__ int s_scan[kTile];
  extern __shared__ int s_wcnt[];  // [kTile/32][E] per-warp counts
  const int tid = threadIdx.x;
  const int tile = blockIdx.x;

  // 1. per expert: total count and the count in the tiles before this one
  //    (a single tile, tile_hist == nullptr, counts its own elements here)
  if (tile_hist == nullptr) {
    for (int e = tid; e < E; e += kTile) {
      s_tot[e] = 0;
      s_start[e] = 0;
    }
    __syncthreads();
    if (tid < N) {
      const int64_t ev = idx[tid];
      if (ev >= 0 && ev < E) atomicAdd(&s_tot[ev], 1);
      else record_error(st, DWDP_ERR_DEVICE_BOUNDS, 100, tid);
    }
  } else {
    for (int e = tid; e < E; e += kTile) {
      int pre = 0, tot = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int v = tile_hist[(int64_t)t * E + e];
        tot += v;
        pre += (t < tile) ? v : 0;
      }
      s_tot[e] = tot;
      s_start[e] = pre;
    }
  }
  for (int i = tid; i < (kTile / 32) * E; i += kTile) s_wcnt[i] = 0;
  __syncthreads();

  // 2. exclusive scan of totals over experts (chunks of kTile)
  int carry = 0;
  for (int base = 0; base < E; base += kTile) {
    const int e = base + tid;
    const int v = (e < E) ? s_tot[e] : 0;
    s_scan[tid] = v;
    __syncthreads();
    for (int off = 1; off < kTile; off <<= 1) {
      const int add = (tid >= off) ? s_scan[tid - off] : 0;
      __syncthreads();
      s_scan[tid] += add;
      __syncthreads();
    }
    const int incl = s_scan[tid];
    if (e < E) {
      const int excl = carry + incl - v;
      s_start[e] += excl;
      if (tile == 0) {
        counts[e] = v;
        offsets[e] = excl;
        if (e == E - 1) offsets[E] = excl + v;
      }
    }
    carry += s_scan[kTile - 1];
    __syncthreads();
  }

  // 3. stable rank inside the tile: rank in warp from the match mask, plus the
  //    counts of the same expert in lower warps of this tile
  const int64_t i = (int64_t)tile * kTile + tid;
  const int lane = tid & 31, warp = tid >> 5;
  int e = -1;
  if (i < N) {
    const int64_t ev = idx[i];
    e = (ev >= 0 && ev < E) ? (int)ev : -1;
  }
  const unsigned mask = __match_any_sync(0xffffffffu, e);
  const int rank_in_warp = __popc(mask & ((1u << lane) - 1u));
  if (e >= 0 && rank_in_warp == 0) s_wcnt[warp * E + e] = __popc(mask);
  __syncthreads();
  if (e >= 0) {
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_wcnt[w * E + e];
    const int64_t d = (int64_t)s_start[e] + before + rank_in_warp;
    perm[d] = i;
    inv[i] = d;
    ids[d] = e;
    tok[d] = i / K;
    packed_w[d] = wts[i];
  }
}

// packed[d, :] = hidden[tok[d], :], bf16 rows, one warp per row.
__global__ void __launch_bounds__(256)
gather_rows_kernel(const __nv_bfloat16* __restrict__ hidden, const int64_t* __restrict__ tok,
                   int64_t N, int H, int64_t T, __nv_bfloat16* __restrict__ packed,
                   DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  const int64_t d = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (d >= N) return;
  const int lane = threadIdx.x & 31;
  const int64_t t = tok[d];
  if (t < 0 || t >= T) {
    if (lane == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 101, (int)d);
    return;
  }
  const __nv_bfloat16* src = hidden + t * H;
  __nv_bfloat16* dst = packed + d * H;
  if ((H & 7) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int c = lane; c < H / 8; c += 32) d4[c] = __ldg(s4 + c);
  } else {
    for (int c = lane; c < H; c += 32) dst[c] = src[c];
  }
}

}  // namespace dwdp

using namespace dwdp;

extern "C" int dwdp_gather_rows_launch(const void* hidden, const int64_t* tok, int64_t N, int H, int64_t T,
                                       void* packed, int* status, cudaStream_t stream) {
  if (N <= 0) return DWDP_OK;
  return launch_chained(gather_rows_kernel, dim3((unsigned)((N + 7) / 8)), dim3(256), 0, stream, 1u,
                        (const __nv_bfloat16*)hidden, tok, N, H, T, (__nv_bfloat16*)packed,
                        reinterpret_cast<DeviceStatus*>(status)) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

extern "C" size_t dwdp_dispatch_scratch_bytes(int64_t num_tokens, int top_k, int num_experts) {
  const int64_t N = num_tokens * top_k;
  const int64_t ntiles = (N + kTile - 1) / kTile;
  return (size_t)((ntiles > 0 ? ntiles : 1) * num_experts * sizeof(int) + 256);
}

extern "C" int dwdp_dispatch_launch(const int64_t* idx, const void* wts, int weight_dtype,
                                    int64_t T, int K, int E, int64_t* counts, int64_t* offsets,
                                    int64_t* perm, int64_t* inv, int64_t* ids, int64_t* tok,
                                    void* packed_w, const void* hidden, int H, void* packed_hidden,
                                    void* scratch, int* status, cudaStream_t stream) {
  if (E <= 0 || E > kMaxExperts || K <= 0 || T < 0) return DWDP_ERR_INVALID_ARGUMENT;
  const int64_t N = T * K;
  DeviceStatus* st = reinterpret_cast<DeviceStatus*>(status);
  if (N == 0) {
    if (cudaMemsetAsync(counts, 0, sizeof(int64_t) * E, stream) != cudaSuccess) return DWDP_ERR_CUDA;
    if (cudaMemsetAsync(offsets, 0, sizeof(int64_t) * (E + 1), stream) != cudaSuccess)
      return DWDP_ERR_CUDA;
    return DWDP_OK;
  }
  const int ntiles = (int)((N + kTile - 1) / kTile);
  // one tile (T * K <= 256, decode batches): the scatter CTA builds its own histogram
  int* tile_hist = ntiles > 1 ? reinterpret_cast<int*>(scratch) : nullptr;
  if (ntiles > 1 && launch_chained(dispatch_hist_kernel, dim3(ntiles), dim3(kTile), 0, stream, 1u, idx, N, E,
                                   tile_hist, st) != cudaSuccess)
    return DWDP_ERR_CUDA;
  const size_t smem = sizeof(int) * (size_t)(kTile / 32) * E;
  if (weight_dtype == DWDP_DTYPE_F32) {
    if (launch_chained(dispatch_scatter_kernel<float>, dim3(ntiles), dim3(kTile), smem, stream, 1u, idx,
                       (const float*)wts, N, K, E, ntiles, (const int*)tile_hist, counts, offsets, perm, inv, ids,
                       tok, (float*)packed_w, st) != cudaSuccess)
      return DWDP_ERR_CUDA;
  } else if (weight_dtype == DWDP_DTYPE_BF16 || weight_dtype == DWDP_DTYPE_F16) {
    if (launch_chained(dispatch_scatter_kernel<uint16_t>, dim3(ntiles), dim3(kTile), smem, stream, 1u, idx,
                       (const uint16_t*)wts, N, K, E, ntiles, (const int*)tile_hist, counts, offsets, perm, inv,
                       ids, tok, (uint16_t*)packed_w, st) != cudaSuccess)
      return DWDP_ERR_CUDA;
  } else {
    return DWDP_ERR_UNSUPPORTED;
  }
  if (hidden != nullptr && packed_hidden != nullptr) {
    const int64_t blocks = (N + 7) / 8;
    if (launch_chained(gather_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, 1u,
                       (const __nv_bfloat16*)hidden, (const int64_t*)tok, N, H, T, (__nv_bfloat16*)packed_hidden,
                       st) != cudaSuccess)
      return DWDP_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Allocation-free dispatch. Some callers cannot allocate device memory at the
// moment they dispatch: code running under an allocator that forbids new
// allocations (a serving loop with a fixed memory budget), plugins that only
// receive the tensors of one call, or hosts without a device allocator of their
// own. For them the per-tile histogram scratch lives in this fixed array, which
// every GPU that loads the library holds until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace dwdp {

// 1 MiB: enough for ceil(T*K / 256) * E <= 262144 (e.g. T*K = 65536 with E = 1024).
constexpr size_t kNoAllocScratchInts = 262144;
static __device__ __align__(256) int g_dispatch_scratch[kNoAllocScratchInts];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
int* g_scratch_ptr[kMaxDevices] = {};  // device address of g_dispatch_scratch, per device
}  // namespace

}  // namespace dwdp

extern "C" size_t dwdp_dispatch_noalloc_max_scratch_bytes(void) {
  return dwdp::kNoAllocScratchInts * sizeof(int);
}

// The host-side name g_dispatch_scratch is only a stand-in; the device address
// comes from cudaGetSymbolAddress, looked up once per device with that device
// current (the first call on a device does it, so make that call before any
// stream capture). Nothing in the array has to start at zero: every call first
// writes each histogram entry it later reads. Calls that overlap on the GPU
// (on different streams) share the array and race.
extern "C" int dwdp_dispatch_noalloc_launch(const int64_t* idx, const void* wts, int weight_dtype,
                                            int64_t T, int K, int E, int64_t* counts,
                                            int64_t* offsets, int64_t* perm, int64_t* inv,
                                            int64_t* ids, int64_t* tok, void* packed_w,
                                            const void* hidden, int H, void* packed_hidden,
                                            int* status, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DWDP_ERR_CUDA;
  if (dev < 0 || dev >= dwdp::kMaxDevices) return DWDP_ERR_UNSUPPORTED;
  int* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(dwdp::g_scratch_mu);
    if (dwdp::g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, dwdp::g_dispatch_scratch) != cudaSuccess || p == nullptr)
        return DWDP_ERR_CUDA;
      dwdp::g_scratch_ptr[dev] = static_cast<int*>(p);
    }
    scratch = dwdp::g_scratch_ptr[dev];
  }
  return dwdp_dispatch_launch(idx, wts, weight_dtype, T, K, E, counts, offsets, perm, inv, ids, tok,
                              packed_w, hidden, H, packed_hidden, scratch, status, stream);
}

// Merger: deterministic token-major reduction of the expert-major weighted
// rows (replaces reference_merge, DWDP/merger/kernels/reference.py:6-27, which
// is zeros[T,H].index_add_(0, packed_token_indices, weighted) — atomics on a
// GPU, hence run-to-run nondeterministic there).
//
// Each token's K rows are found through inv[t*K + k] (the destination of
// assignment (t, k)) and summed in ascending row order, which is the order the
// CPU index_add_ visits them. The optional shared-expert rows (the K-split
// partials of the shared down projection, summed in order) are added last
// (DWDP/adapters/qwen15_moe.py:302-319 adds it after the merger). fp32
// accumulation, 16-byte vector loads; one CTA per token, HBM-bound.
#include "common.cuh"

namespace dwdp {

constexpr int kMergeMaxK = 16;
constexpr int kMergeMaxParts = 8;

// 8 bf16 of a 16-byte vector added into acc[0..8)
__device__ __forceinline__ void add8(float (&acc)[8], const uint4& v) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(b[q]);
    acc[2 * q] += f.x;
    acc[2 * q + 1] += f.y;
  }
}

// One CTA per token. Thread 0 sorts the token's K packed rows ascending in
// shared memory; every thread then issues all of its row loads (and the shared
// partials) before summing them in that fixed order, so a token costs about one
// memory latency.
template <typename TOut, int KMAX, int PMAX>
__global__ void __launch_bounds__(256)
merge_kernel(const __nv_bfloat16* __restrict__ weighted, const int64_t* __restrict__ inv,
             const __nv_bfloat16* __restrict__ shared_out, int shared_parts,
             const float* __restrict__ shared_gate, int64_t T, int K, int H,
             int64_t nrows, TOut* __restrict__ out, DeviceStatus* st) {
  griddep_launch();
  __shared__ int64_t s_rows[KMAX];
  __shared__ int s_nk;
  const int64_t t = blockIdx.x;
  griddep_wait();
  if (threadIdx.x == 0) {
    int nk = 0;
    for (int k = 0; k < K; ++k) {
      const int64_t r = inv[t * K + k];
      if (r < 0 || r >= nrows) {
        record_error(st, DWDP_ERR_DEVICE_BOUNDS, 300, (int)t);
        continue;
      }
      int p = nk++;  // insertion into ascending order
      while (p > 0 && s_rows[p - 1] > r) { s_rows[p] = s_rows[p - 1]; --p; }
      s_rows[p] = r;
    }
    s_nk = nk;
  }
  __syncthreads();
  const int nk = s_nk;
  const float* sgate = shared_gate;
  const float sgate_t = sgate != nullptr ? sgate[t] : 1.0f;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 v[KMAX], sv[PMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < nk) v[j] = *reinterpret_cast<const uint4*>(weighted + s_rows[j] * H + c);
#pragma unroll
    for (int sp = 0; sp < PMAX; ++sp)
      if (sp < shared_parts) sv[sp] = *reinterpret_cast<const uint4*>(shared_out + ((int64_t)sp * T + t) * H + c);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < nk) add8(acc, v[j]);
    if (sgate == nullptr) {
#pragma unroll
      for (int sp = 0; sp < PMAX; ++sp)
        if (sp < shared_parts) add8(acc, sv[sp]);
    } else {  // ungated shared partials: out += gate[t] * sum of parts
      float sacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int sp = 0; sp < PMAX; ++sp)
        if (sp < shared_parts) add8(sacc, sv[sp]);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += sgate_t * sacc[q];
    }
    if constexpr (sizeof(TOut) == 2) {
      uint4 o;
      __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) ob[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      *reinterpret_cast<uint4*>(out + t * H + c) = o;
    } else {
      float4* o = reinterpret_cast<float4*>(out + t * H + c);
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

}  // namespace dwdp

using namespace dwdp;

extern "C" int dwdp_merge_launch(const void* weighted, const int64_t* inv, const void* shared_out,
                                 int shared_parts, const float* shared_gate, int64_t T, int K, int H, void* out,
                                 int out_dtype,
                                 int* status,
                                 cudaStream_t stream) {
  if (K <= 0 || K > kMergeMaxK || (H & 7) != 0 || T < 0 || shared_parts < 0) return DWDP_ERR_INVALID_ARGUMENT;
  if (shared_out != nullptr && shared_parts > kMergeMaxParts) return DWDP_ERR_UNSUPPORTED;
  if (T == 0) return DWDP_OK;
  if (shared_out == nullptr) shared_parts = 0;
  DeviceStatus* st = reinterpret_cast<DeviceStatus*>(status);
  const int threads = H / 8 >= 256 ? 256 : ((H / 8 + 31) / 32) * 32;
  // register staging sized to the call: K rows and the shared partials
  auto go = [&](auto kfn, auto* typed_out) {
    return launch_chained(kfn, dim3((unsigned)T), dim3(threads), 0, stream, 1u, (const __nv_bfloat16*)weighted, inv,
                          (const __nv_bfloat16*)shared_out, shared_parts, shared_gate, T, K, H, T * K, typed_out, st);
  };
  const bool f32 = out_dtype == DWDP_DTYPE_F32;
  if (!f32 && out_dtype != DWDP_DTYPE_BF16) return DWDP_ERR_UNSUPPORTED;
  cudaError_t e;
#define DWDP_MERGE(KM, PM)                                                                          \
  e = f32 ? go(merge_kernel<float, KM, PM>, static_cast<float*>(out))                              \
          : go(merge_kernel<__nv_bfloat16, KM, PM>, static_cast<__nv_bfloat16*>(out))
  if (K <= 4 && shared_parts <= 1) DWDP_MERGE(4, 1);
  else if (K <= 4) DWDP_MERGE(4, 8);
  else if (K <= 8 && shared_parts <= 1) DWDP_MERGE(8, 1);
  else if (K <= 8) DWDP_MERGE(8, 8);
  else DWDP_MERGE(16, 8);
#undef DWDP_MERGE
  if (e != cudaSuccess) return DWDP_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

// Streaming multiprocessor copy of expert slabs (the engine's alternative to the copy
// engines, DWDP_COPY_SM): every CTA walks a grid-strided range of 16-byte vectors of each
// listed copy, loading from the source (a peer GPU's memory through an IPC mapping or a
// peer pointer: plain loads, no multicast) and storing into this GPU's staging buffer.
// Loads and stores are streaming (evict-first): the staged slabs are read by the next layer,
// long after the current layer's GEMMs, whose L2-resident weight tiles they must not evict.
// Copy engines take no SMs from the persistent GEMMs, SM copies do; the engine measures
// both (the reference's buffers.cu used cudaMemcpyPeerAsync, i.e. the copy engines).
#include <cuda_runtime.h>

#include <cstdint>

#include "dwdp_b200.h"

namespace dwdp {

// 128 threads: small enough to sit beside a persistent GEMM CTA on the same SM
constexpr int kCopyThreads = 128;
constexpr int kCopyUnroll = 4;  // 16-byte loads in flight per thread per step

__global__ void __launch_bounds__(kCopyThreads) peer_copy_kernel(dwdp_copy_list list) {
  const size_t tid = (size_t)blockIdx.x * kCopyThreads + threadIdx.x;
  const size_t nthreads = (size_t)gridDim.x * kCopyThreads;
  for (int c = 0; c < list.n; ++c) {
    const uint4* __restrict__ src = reinterpret_cast<const uint4*>(list.src[c]);
    uint4* __restrict__ dst = reinterpret_cast<uint4*>(list.dst[c]);
    const size_t nv = list.bytes[c] / 16;
    size_t i = tid;
    // kCopyUnroll loads issued before their stores
    for (; i + (kCopyUnroll - 1) * nthreads < nv; i += kCopyUnroll * nthreads) {
      uint4 v[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) v[u] = __ldcs(src + i + u * nthreads);
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) __stcs(dst + i + u * nthreads, v[u]);
    }
    for (; i < nv; i += nthreads) __stcs(dst + i, __ldcs(src + i));
    // a ragged tail (sizes not a multiple of 16) byte by byte
    const size_t tail = list.bytes[c] - nv * 16;
    if (tid < tail)
      reinterpret_cast<uint8_t*>(list.dst[c])[nv * 16 + tid] =
          reinterpret_cast<const uint8_t*>(list.src[c])[nv * 16 + tid];
  }
}

}  // namespace dwdp

extern "C" int dwdp_peer_copy_sm(const dwdp_copy_list* list, int ctas, void* stream) {
  if (list == nullptr || list->n < 0 || list->n > DWDP_COPY_LIST_MAX || ctas <= 0)
    return DWDP_ERR_INVALID_ARGUMENT;
  for (int c = 0; c < list->n; ++c) {
    if (list->bytes[c] == 0) continue;
    if (list->src[c] == nullptr || list->dst[c] == nullptr) return DWDP_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(list->src[c]) | reinterpret_cast<uintptr_t>(list->dst[c])) & 15)
      return DWDP_ERR_INVALID_ARGUMENT;
  }
  if (list->n == 0) return DWDP_OK;
  dwdp::peer_copy_kernel<<<ctas, dwdp::kCopyThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*list);
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

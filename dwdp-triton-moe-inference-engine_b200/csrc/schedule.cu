// Scheduler: deterministic ascending-expert round-robin schedule
// (DWDP/scheduler/ops/round_robin.py:8-80) computed on device. The reference
// uses torch.nonzero (an implicit device->host sync) to size its outputs; here
// the outputs are fixed at E entries, rows past num_active hold -1, and the
// active count is a device scalar, so the schedule is CUDA-graph capturable.
#include "common.cuh"

namespace dwdp {

__global__ void __launch_bounds__(1024)
schedule_kernel(const int64_t* __restrict__ counts, const int64_t* __restrict__ offsets, int E,
                int stream_count, int64_t* __restrict__ queue, int64_t* __restrict__ starts,
                int64_t* __restrict__ ends, int64_t* __restrict__ active_counts,
                int64_t* __restrict__ priority, int64_t* __restrict__ stream_ids,
                int64_t* __restrict__ num_active) {
  __shared__ int s_scan[1024];
  __shared__ int s_total;
  const int tid = threadIdx.x;
  int carry = 0;
  for (int e0 = 0; e0 < E; e0 += 1024) {
    const int e = e0 + tid;
    const int act = (e < E && counts[e] > 0) ? 1 : 0;
    s_scan[tid] = act;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
      const int add = tid >= o ? s_scan[tid - o] : 0;
      __syncthreads();
      s_scan[tid] += add;
      __syncthreads();
    }
    if (act) {
      const int pos = carry + s_scan[tid] - 1;
      queue[pos] = e;
      starts[pos] = offsets[e];
      ends[pos] = offsets[e + 1];
      active_counts[pos] = counts[e];
      priority[pos] = pos;
      stream_ids[pos] = pos % stream_count;
    }
    if (tid == 1023) s_total = carry + s_scan[1023];
    __syncthreads();
    carry = s_total;
    __syncthreads();
  }
  for (int i = carry + tid; i < E; i += 1024) {
    queue[i] = -1;
    starts[i] = -1;
    ends[i] = -1;
    active_counts[i] = -1;
    priority[i] = -1;
    stream_ids[i] = -1;
  }
  if (tid == 0) *num_active = carry;
}

}  // namespace dwdp

using namespace dwdp;

extern "C" int dwdp_schedule_launch(const int64_t* counts, const int64_t* offsets, int E,
                                    int stream_count, int64_t* queue, int64_t* starts,
                                    int64_t* ends, int64_t* active_counts, int64_t* priority,
                                    int64_t* stream_ids, int64_t* num_active,
                                    cudaStream_t stream) {
  if (E <= 0 || stream_count <= 0) return DWDP_ERR_INVALID_ARGUMENT;
  schedule_kernel<<<1, 1024, 0, stream>>>(counts, offsets, E, stream_count, queue, starts, ends,
                                          active_counts, priority, stream_ids, num_active);
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

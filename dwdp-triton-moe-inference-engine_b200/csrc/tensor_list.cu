// TensorList: the structure-of-arrays handle set of the active experts
// (DWDP/executor/tensor_list.py:29-228), filled on the device from an execution
// plan. The reference fills it on the host (one pass over the plan, a pinned
// H2D copy and a stream sync); here one CTA compacts the plan's rows with
// count > 0 and writes every field, so no count reaches the host and the fill
// can sit inside a CUDA graph. The grouped GEMM then reads the TensorList's
// own pointer / offset / count rows as its expert group (dwdp_grouped_moe).
#include "common.cuh"

namespace dwdp {

constexpr int kTlThreads = 1024;

struct TlBuildParams {
  const int64_t* queue;     // plan rows: expert id (-1 = padding)
  const int64_t* starts;    // first packed row of the expert
  const int64_t* counts;    // rows of the expert (<= 0 = skipped)
  const int64_t* priority;  // may be null: row position
  const int64_t* streams;   // may be null: 0
  int plan_len;
  const int64_t* w13;       // [E] packed gate/up slab per expert
  const int64_t* w2;        // [E] packed down tiles
  const int64_t* s13;       // [E] gate/up scales (0 for bf16)
  const int64_t* s2;        // [E] down scales
  int num_experts;
  dwdp_tensor_list_bases b;
  int64_t capacity;
  int64_t* fields;          // [DWDP_TL_ROWS][capacity]
  int64_t* meta;            // [2]: size, max tokens of one entry
  DeviceStatus* st;
};

__global__ void __launch_bounds__(kTlThreads) tensor_list_build_kernel(const TlBuildParams p) {
  __shared__ int s_scan[kTlThreads];
  __shared__ int s_total;
  __shared__ int s_max;
  const int tid = threadIdx.x;
  const int64_t cap = p.capacity;
  if (tid == 0) s_max = 0;
  int carry = 0;
  for (int r0 = 0; r0 < p.plan_len; r0 += kTlThreads) {
    const int r = r0 + tid;
    int64_t e = -1, cnt = 0;
    if (r < p.plan_len) {
      e = p.queue[r];
      cnt = p.counts[r];
    }
    int act = (e >= 0 && cnt > 0) ? 1 : 0;
    if (act && e >= p.num_experts) {
      record_error(p.st, DWDP_ERR_DEVICE_BOUNDS, 900, (int)e);
      act = 0;
    }
    s_scan[tid] = act;
    __syncthreads();
    for (int o = 1; o < kTlThreads; o <<= 1) {
      const int add = tid >= o ? s_scan[tid - o] : 0;
      __syncthreads();
      s_scan[tid] += add;
      __syncthreads();
    }
    const int pos = carry + s_scan[tid] - 1;
    if (act && pos < cap) {
      const int64_t off = p.starts[r];
      int64_t* f = p.fields + pos;
      f[DWDP_TL_INPUT_PTRS * cap] = (int64_t)p.b.input;
      f[DWDP_TL_TOKEN_INDEX_PTRS * cap] = (int64_t)p.b.token_index;
      f[DWDP_TL_ROUTING_WEIGHT_PTRS * cap] = (int64_t)p.b.routing_weights;
      f[DWDP_TL_GATE_WEIGHT_PTRS * cap] = p.w13[e];
      f[DWDP_TL_UP_WEIGHT_PTRS * cap] = p.w13[e];  // gate and up share one packed slab
      f[DWDP_TL_DOWN_WEIGHT_PTRS * cap] = p.w2[e];
      f[DWDP_TL_INTERMEDIATE_PTRS * cap] =
          p.b.intermediate ? (int64_t)p.b.intermediate + off * p.b.intermediate_row_bytes : 0;
      f[DWDP_TL_OUTPUT_PTRS * cap] = p.b.output ? (int64_t)p.b.output + off * p.b.output_row_bytes : 0;
      f[DWDP_TL_WEIGHTED_OUTPUT_PTRS * cap] =
          p.b.weighted_output ? (int64_t)p.b.weighted_output + off * p.b.weighted_row_bytes : 0;
      f[DWDP_TL_QUANTIZATION_PTRS * cap] = p.s13 ? p.s13[e] : 0;
      f[DWDP_TL_EXPERT_IDS * cap] = e;
      f[DWDP_TL_TOKEN_OFFSETS * cap] = off;
      f[DWDP_TL_TOKEN_COUNTS * cap] = cnt;
      f[DWDP_TL_M * cap] = cnt;
      f[DWDP_TL_N * cap] = p.b.n;
      f[DWDP_TL_K * cap] = p.b.k;
      f[DWDP_TL_INTERMEDIATE_N * cap] = p.b.intermediate_n;
      f[DWDP_TL_INPUT_LD * cap] = p.b.input_ld;
      f[DWDP_TL_GATE_LD * cap] = p.b.gate_ld;
      f[DWDP_TL_UP_LD * cap] = p.b.up_ld;
      f[DWDP_TL_DOWN_LD * cap] = p.b.down_ld;
      f[DWDP_TL_OUTPUT_LD * cap] = p.b.output_ld;
      f[DWDP_TL_DTYPE_CODES * cap] = p.b.dtype_code;
      f[DWDP_TL_WORKSPACE_INDICES * cap] = pos;
      f[DWDP_TL_EXECUTION_PRIORITIES * cap] = p.priority ? p.priority[r] : r;
      f[DWDP_TL_STREAM_IDS * cap] = p.streams ? p.streams[r] : 0;
      f[DWDP_TL_DOWN_QUANTIZATION_PTRS * cap] = p.s2 ? p.s2[e] : 0;
      atomicMax(&s_max, cnt > 0x7fffffff ? 0x7fffffff : (int)cnt);
    } else if (act) {
      record_error(p.st, DWDP_ERR_CAPACITY, 901, pos);
    }
    if (tid == kTlThreads - 1) s_total = carry + s_scan[kTlThreads - 1];
    __syncthreads();
    carry = s_total;
    __syncthreads();
  }
  const int size = carry < cap ? carry : (int)cap;
  // Entries past `size` read as empty experts (count 0, null pointers), so a grouped
  // launch over all `capacity` entries skips them without knowing `size`.
  for (int64_t i = size + tid; i < cap; i += kTlThreads) {
    for (int fld = 0; fld < DWDP_TL_ROWS; ++fld) p.fields[fld * cap + i] = 0;
    p.fields[DWDP_TL_EXPERT_IDS * cap + i] = -1;
  }
  if (tid == 0) {
    p.meta[0] = size;
    p.meta[1] = s_max;
  }
}

}  // namespace dwdp

using namespace dwdp;

extern "C" int dwdp_tensor_list_build_launch(const int64_t* queue, const int64_t* starts, const int64_t* counts,
                                             const int64_t* priority, const int64_t* streams, int plan_len,
                                             const dwdp_expert_group* experts, const dwdp_tensor_list_bases* bases,
                                             int64_t capacity, int64_t* fields, int64_t* meta, int* status,
                                             cudaStream_t stream) {
  TlBuildParams p{};
  p.queue = queue; p.starts = starts; p.counts = counts; p.priority = priority; p.streams = streams;
  p.plan_len = plan_len;
  p.w13 = reinterpret_cast<const int64_t*>(experts->w13);
  p.w2 = reinterpret_cast<const int64_t*>(experts->w2);
  p.s13 = reinterpret_cast<const int64_t*>(experts->s13);
  p.s2 = reinterpret_cast<const int64_t*>(experts->s2);
  p.num_experts = experts->num_experts;
  p.b = *bases;
  p.capacity = capacity; p.fields = fields; p.meta = meta;
  p.st = reinterpret_cast<DeviceStatus*>(status);
  tensor_list_build_kernel<<<1, kTlThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

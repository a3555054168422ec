// Router: fused logits tile + top-k + softmax-over-k + renormalisation, plus the
// optional sigmoid shared-expert gate.
//
// Semantics follow DWDP/router/linear.py:38-44 (logits = x W^T + b, times
// score_scale) and DWDP/router/kernels/fused.py:8-42 (top-k over the logits,
// softmax over the k selected, renormalise by sum.clamp_min(eps), k == 1 ->
// weight 1). Arithmetic is fp32 throughout. Top-k ties resolve to the lower
// expert id and slots come out in descending logit order.
//
// Layout: one CTA of 256 threads owns 32 tokens. x[32][64] and W[E'][64] chunks
// (E' = E + 1 when the shared gate row is appended) are staged in shared memory
// as fp32; thread (token = tid/8, lane group g = tid%8) accumulates experts
// g, g+8, ... in registers. The router reads E*H*2 bytes of weights per CTA from
// L2 and its FLOPs are a rounding error next to the expert GEMMs.
#include "common.cuh"

namespace dwdp {

constexpr int kRouterTok = 32;
constexpr int kRouterH = 64;
constexpr int kRouterThreads = 256;
constexpr int kRouterMaxRows = 264;  // E <= 256 plus the shared-gate row, rounded to 8

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename TX, typename TW>
__global__ void __launch_bounds__(kRouterThreads)
router_topk_kernel(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ bias,
                   const TW* __restrict__ gate_w, int T, int H, int E, int K, float score_scale,
                   int renorm, float eps, float* __restrict__ logits_out, float* __restrict__ probs,
                   int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                   float* __restrict__ shared_gate) {
  extern __shared__ float sm[];
  const int rows = E + (gate_w != nullptr ? 1 : 0);
  float* xs = sm;                                // [32][kRouterH+1]
  float* ws = xs + kRouterTok * (kRouterH + 1);  // [rows][kRouterH+1]
  float* ls = ws + rows * (kRouterH + 1);        // [32][rows+1] logits
  const int t0 = blockIdx.x * kRouterTok;
  const int tid = threadIdx.x;
  const int my_tok = tid >> 3;
  const int g = tid & 7;
  const int nper = (rows + 7) >> 3;

  float acc[kRouterMaxRows / 8];
#pragma unroll
  for (int i = 0; i < kRouterMaxRows / 8; ++i) acc[i] = 0.f;

  for (int h0 = 0; h0 < H; h0 += kRouterH) {
    const int hn = min(kRouterH, H - h0);
    for (int i = tid; i < kRouterTok * kRouterH; i += kRouterThreads) {
      const int tt = i / kRouterH, hh = i % kRouterH;
      float v = 0.f;
      if (t0 + tt < T && hh < hn) v = to_f32(x[(int64_t)(t0 + tt) * H + h0 + hh]);
      xs[tt * (kRouterH + 1) + hh] = v;
    }
    for (int i = tid; i < rows * kRouterH; i += kRouterThreads) {
      const int e = i / kRouterH, hh = i % kRouterH;
      float v = 0.f;
      if (hh < hn) v = (e < E) ? to_f32(w[(int64_t)e * H + h0 + hh]) : to_f32(gate_w[h0 + hh]);
      ws[e * (kRouterH + 1) + hh] = v;
    }
    __syncthreads();
    const float* xr = xs + my_tok * (kRouterH + 1);
    for (int hh = 0; hh < hn; ++hh) {
      const float xv = xr[hh];
#pragma unroll
      for (int i = 0; i < kRouterMaxRows / 8; ++i) {
        const int e = g + 8 * i;
        if (i < nper && e < rows) acc[i] = fmaf(xv, ws[e * (kRouterH + 1) + hh], acc[i]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < kRouterMaxRows / 8; ++i) {
    const int e = g + 8 * i;
    if (i < nper && e < rows) {
      float v = acc[i];
      if (e < E) {
        if (bias != nullptr) v += bias[e];
        v *= score_scale;
      }
      ls[my_tok * (rows + 1) + e] = v;
    }
  }
  __syncthreads();

  // one warp per token: top-k by repeated arg-max (ties -> lower id)
  const int warp = tid >> 5, lane = tid & 31;
  for (int tt = warp; tt < kRouterTok; tt += kRouterThreads / 32) {
    const int t = t0 + tt;
    if (t >= T) break;
    const float* lr = ls + tt * (rows + 1);
    if (logits_out != nullptr)
      for (int e = lane; e < E; e += 32) logits_out[(int64_t)t * E + e] = lr[e];
    if (shared_gate != nullptr && gate_w != nullptr && lane == 0)
      shared_gate[t] = 1.0f / (1.0f + expf(-lr[E]));
    uint32_t taken = 0;  // bit j: this lane's expert lane + 32*j already selected
    float sel_v[16];
    int sel_i[16];
    for (int k = 0; k < K; ++k) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int j = 0; lane + 32 * j < E; ++j) {
        if (taken & (1u << j)) continue;
        const int e = lane + 32 * j;
        const float v = lr[e];
        if (bi == 0x7fffffff || v > best) { best = v; bi = e; }  // ascending e: ties keep lower id
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > best || (ov == best && oi < bi))) {
          best = ov;
          bi = oi;
        }
      }
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      sel_v[k] = best;
      sel_i[k] = bi;
    }
    if (lane == 0) {
      // softmax over the k selected logits, fp32 (max-subtracted)
      const float m = sel_v[0];
      float p[16];
      float s = 0.f;
      for (int k = 0; k < K; ++k) { p[k] = expf(sel_v[k] - m); s += p[k]; }
      float psum = 0.f;
      for (int k = 0; k < K; ++k) { p[k] = p[k] / s; psum += p[k]; }
      const float den = fmaxf(psum, eps);
      for (int k = 0; k < K; ++k) {
        const int64_t o = (int64_t)t * K + k;
        idx_out[o] = sel_i[k];
        if (probs != nullptr) probs[o] = p[k];
        w_out[o] = (K == 1) ? 1.0f : (renorm ? p[k] / den : p[k]);
      }
    }
  }
}

}  // namespace dwdp

using namespace dwdp;

extern "C" int dwdp_router_launch(const void* hidden, int hidden_dtype, const void* weight,
                                  int weight_dtype, const float* bias,
                                  const void* shared_gate_weight, int64_t T, int H, int E, int K,
                                  float score_scale, int renorm, float eps, float* logits,
                                  float* probs, int64_t* idx, float* topk_w, float* shared_gate,
                                  cudaStream_t stream) {
  const int rows = E + (shared_gate_weight != nullptr ? 1 : 0);
  const size_t smem = sizeof(float) * ((size_t)kRouterTok * (kRouterH + 1) +
                                       (size_t)rows * (kRouterH + 1) + (size_t)kRouterTok * (rows + 1));
  const int grid = (int)((T + kRouterTok - 1) / kRouterTok);
  if (grid == 0) return DWDP_OK;
#define DWDP_LAUNCH_ROUTER(TX, TW)                                                                  \
  do {                                                                                              \
    auto kfn = router_topk_kernel<TX, TW>;                                                          \
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=       \
        cudaSuccess)                                                                                \
      return DWDP_ERR_CUDA;                                                                         \
    kfn<<<grid, kRouterThreads, smem, stream>>>(                                                    \
        (const TX*)hidden, (const TW*)weight, bias, (const TW*)shared_gate_weight, (int)T, H, E, K, \
        score_scale, renorm, eps, logits, probs, idx, topk_w, shared_gate);                         \
  } while (0)
  if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_BF16)
    DWDP_LAUNCH_ROUTER(__nv_bfloat16, __nv_bfloat16);
  else if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_F32)
    DWDP_LAUNCH_ROUTER(__nv_bfloat16, float);
  else if (hidden_dtype == DWDP_DTYPE_F32 && weight_dtype == DWDP_DTYPE_F32)
    DWDP_LAUNCH_ROUTER(float, float);
  else if (hidden_dtype == DWDP_DTYPE_F32 && weight_dtype == DWDP_DTYPE_BF16)
    DWDP_LAUNCH_ROUTER(float, __nv_bfloat16);
  else
    return DWDP_ERR_UNSUPPORTED;
#undef DWDP_LAUNCH_ROUTER
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

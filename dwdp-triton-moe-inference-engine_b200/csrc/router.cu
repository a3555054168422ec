// Router: fused logits tile + top-k + softmax-over-k + renormalisation, plus the
// optional sigmoid shared-expert gate.
//
// Semantics follow DWDP/router/linear.py:38-44 (logits = x W^T + b, times
// score_scale) and DWDP/router/kernels/fused.py:8-42 (top-k over the logits,
// softmax over the k selected, renormalise by sum.clamp_min(eps), k == 1 ->
// weight 1). Arithmetic is fp32 throughout. Top-k ties resolve to the lower
// expert id and slots come out in descending logit order.
//
// Layout: see router_topk_kernel below.
#include "common.cuh"

namespace dwdp {

constexpr int kRouterThreads = 256;  // 8 warps

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// 8 consecutive elements -> fp32 (16 bytes of bf16 or 32 bytes of fp32)
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(b[q]);
    v[2 * q] = f.x;
    v[2 * q + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// One CTA owns TOK tokens. Their rows are staged in shared memory as fp32
// (TOK x H). Warp w computes the logits of experts w, w+8, ...: lanes split H in
// 8-element slices (16-byte weight loads straight from L2/HBM, each weight slice
// reused for all TOK tokens from registers), then a shuffle reduction per
// (expert, token). Logits land in shared memory for the top-k phase, in which one
// warp handles one token.
template <typename TX, typename TW, int TOK>
__global__ void __launch_bounds__(kRouterThreads)
router_topk_kernel(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ bias,
                   const TW* __restrict__ gate_w, int T, int H, int E, int K, float score_scale,
                   int renorm, float eps, float* __restrict__ logits_out, float* __restrict__ probs,
                   int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                   float* __restrict__ shared_gate) {
  extern __shared__ float sm[];
  const int rows = E + (gate_w != nullptr ? 1 : 0);
  float* xs = sm;                   // [TOK][H]
  float* ls = xs + (size_t)TOK * H;  // [TOK][rows + 1]
  const int t0 = blockIdx.x * TOK;
  const int ntok = min(TOK, T - t0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // stage x rows (8 elements per step, independent loads)
  const int h8 = H >> 3;
  for (int i = tid; i < TOK * h8; i += kRouterThreads) {
    const int tt = i / h8, c = (i - tt * h8) * 8;
    float v[8];
    if (tt < ntok) {
      load8(x + (int64_t)(t0 + tt) * H + c, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    float4* dst = reinterpret_cast<float4*>(xs + tt * H + c);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();

  for (int e = warp; e < rows; e += kRouterThreads / 32) {
    const TW* wr = (e < E) ? w + (int64_t)e * H : gate_w;
    float acc[TOK];
#pragma unroll
    for (int tt = 0; tt < TOK; ++tt) acc[tt] = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float wv[8];
      load8(wr + c, wv);
#pragma unroll
      for (int tt = 0; tt < TOK; ++tt) {
        const float4 a = *reinterpret_cast<const float4*>(xs + tt * H + c);
        const float4 b = *reinterpret_cast<const float4*>(xs + tt * H + c + 4);
        float s = acc[tt];
        s = fmaf(a.x, wv[0], s); s = fmaf(a.y, wv[1], s); s = fmaf(a.z, wv[2], s); s = fmaf(a.w, wv[3], s);
        s = fmaf(b.x, wv[4], s); s = fmaf(b.y, wv[5], s); s = fmaf(b.z, wv[6], s); s = fmaf(b.w, wv[7], s);
        acc[tt] = s;
      }
    }
#pragma unroll
    for (int tt = 0; tt < TOK; ++tt) {
      float v = acc[tt];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) {
        if (e < E) {
          if (bias != nullptr) v += bias[e];
          v *= score_scale;
        }
        ls[tt * (rows + 1) + e] = v;
      }
    }
  }
  __syncthreads();

  // one warp per token: top-k by repeated arg-max (ties -> lower id)
  for (int tt = warp; tt < ntok; tt += kRouterThreads / 32) {
    const int t = t0 + tt;
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
  if (T == 0) return DWDP_OK;
  if (H % 8 != 0) return DWDP_ERR_INVALID_ARGUMENT;
  const int rows = E + (shared_gate_weight != nullptr ? 1 : 0);
  // tokens per CTA: as many as fit 160 KB of staged fp32 rows (and no more than needed)
  int tok = 32;
  while (tok > 8 && ((size_t)tok * H * 4 > 160 * 1024 || tok / 2 >= T)) tok /= 2;
  if ((size_t)tok * H * 4 > 200 * 1024) return DWDP_ERR_UNSUPPORTED;
  const size_t smem = sizeof(float) * ((size_t)tok * H + (size_t)tok * (rows + 1));
  const int grid = (int)((T + tok - 1) / tok);
#define DWDP_LAUNCH_ROUTER(TX, TW, TOKN)                                                             \
  do {                                                                                               \
    auto kfn = router_topk_kernel<TX, TW, TOKN>;                                                     \
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=        \
        cudaSuccess)                                                                                 \
      return DWDP_ERR_CUDA;                                                                          \
    kfn<<<grid, kRouterThreads, smem, stream>>>(                                                     \
        (const TX*)hidden, (const TW*)weight, bias, (const TW*)shared_gate_weight, (int)T, H, E, K,  \
        score_scale, renorm, eps, logits, probs, idx, topk_w, shared_gate);                          \
  } while (0)
#define DWDP_ROUTER_TOK(TX, TW)                      \
  do {                                               \
    if (tok == 32) DWDP_LAUNCH_ROUTER(TX, TW, 32);   \
    else if (tok == 16) DWDP_LAUNCH_ROUTER(TX, TW, 16); \
    else DWDP_LAUNCH_ROUTER(TX, TW, 8);              \
  } while (0)
  if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_BF16)
    DWDP_ROUTER_TOK(__nv_bfloat16, __nv_bfloat16);
  else if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_F32)
    DWDP_ROUTER_TOK(__nv_bfloat16, float);
  else if (hidden_dtype == DWDP_DTYPE_F32 && weight_dtype == DWDP_DTYPE_F32)
    DWDP_ROUTER_TOK(float, float);
  else if (hidden_dtype == DWDP_DTYPE_F32 && weight_dtype == DWDP_DTYPE_BF16)
    DWDP_ROUTER_TOK(float, __nv_bfloat16);
  else
    return DWDP_ERR_UNSUPPORTED;
#undef DWDP_ROUTER_TOK
#undef DWDP_LAUNCH_ROUTER
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

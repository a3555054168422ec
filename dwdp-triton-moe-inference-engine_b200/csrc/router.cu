// Router: fused logits tile + top-k + softmax-over-k + renormalisation, plus the
// optional sigmoid shared-expert gate.
//
// Semantics follow DWDP/router/linear.py:38-44 (logits = x W^T + b, times
// score_scale) and DWDP/router/kernels/fused.py:8-42 (top-k over the logits,
// softmax over the k selected, renormalise by sum.clamp_min(eps), k == 1 ->
// weight 1). Arithmetic is fp32 throughout. Top-k ties resolve to the lower
// expert id and slots come out in descending logit order.
//
// bf16 inputs with E <= 256: ONE launch (router_fused_kernel). Otherwise two:
// the logits (router_logits_mma_kernel on the tensor cores for bf16 inputs,
// router_logits_kernel on the CUDA cores for fp32 inputs) and
// router_topk_kernel (one warp per token).
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

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

// Logits: grid (token tiles of TOK, expert groups of 8). The CTA stages its TOK
// token rows in shared memory as bf16; warp w computes expert (8*blockIdx.y + w)
// for all TOK tokens: each lane owns 8-element slices of H, issues all of its
// 16-byte weight loads for the row up front (kMaxSlices in flight), then
// multiplies them against the staged tokens, and a shuffle reduction finishes
// each (expert, token) dot product. One warp computes each logit: deterministic.
constexpr int kMaxSlices = 8;  // H <= 8 * 256 per pass; larger H loops over passes

template <typename TX, typename TW, int TOK>
__global__ void __launch_bounds__(kRouterThreads)
router_logits_kernel(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ bias,
                     const TW* __restrict__ gate_w, int T, int H, int E, float score_scale,
                     float* __restrict__ logits, float* __restrict__ gate_logit) {
  griddep_launch();
  griddep_wait();
  extern __shared__ __align__(16) uint8_t xs_raw[];
  TX* xs = reinterpret_cast<TX*>(xs_raw);  // [TOK][H] in the input dtype (exact)
  const int t0 = blockIdx.x * TOK;
  const int ntok = min(TOK, T - t0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows = E + (gate_w != nullptr ? 1 : 0);
  const int h8 = H >> 3;
  for (int i = tid; i < TOK * h8; i += kRouterThreads) {
    const int tt = i / h8, c = (i - tt * h8) * 8;
    constexpr int kVec = (int)(8 * sizeof(TX) / 16);  // 16-byte vectors per 8 elements
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(t0 + tt) * H + c);
    uint4* dst = reinterpret_cast<uint4*>(xs + tt * H + c);
#pragma unroll
    for (int q = 0; q < kVec; ++q) dst[q] = (tt < ntok) ? src[q] : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const int e = blockIdx.y * 8 + warp;
  if (e >= rows) return;
  const TW* wr = (e < E) ? w + (int64_t)e * H : gate_w;
  float acc[TOK];
#pragma unroll
  for (int tt = 0; tt < TOK; ++tt) acc[tt] = 0.f;
  for (int base = 0; base < H; base += 256 * kMaxSlices) {
    float wv[kMaxSlices][8];
#pragma unroll
    for (int j = 0; j < kMaxSlices; ++j) {
      const int c = base + (j * 32 + lane) * 8;
      if (c < H) {
        load8(wr + c, wv[j]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) wv[j][q] = 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < kMaxSlices; ++j) {
      const int c = base + (j * 32 + lane) * 8;
      if (c >= H) break;
#pragma unroll
      for (int tt = 0; tt < TOK; ++tt) {
        float xv[8];
        load8(xs + tt * H + c, xv);
        float s = acc[tt];
#pragma unroll
        for (int q = 0; q < 8; ++q) s = fmaf(xv[q], wv[j][q], s);
        acc[tt] = s;
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < TOK; ++tt) {
    float v = acc[tt];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0 && tt < ntok) {
      if (e < E) {
        if (bias != nullptr) v += bias[e];
        logits[(int64_t)(t0 + tt) * E + e] = v * score_scale;
      } else {
        gate_logit[t0 + tt] = v;
      }
    }
  }
}

// bf16 x bf16 logits on the tensor cores (mma.sync m16n8k16, fp32 accumulate;
// bf16 products are exact in fp32, so this equals the fp32 CUDA-core result up to
// summation order). A CTA owns 16 tokens x 32 experts (4 n-tiles of 8); its 8
// warps split K (warp w takes the 16-wide K steps with index % 8 == w), so each
// warp has all of its fragment loads in flight at once, and the 8 partial tiles
// are summed through shared memory in a fixed order (deterministic).
constexpr int kMmaTok = 16;
constexpr int kMmaExp = 32;
constexpr int kMmaWarps = 8;

__device__ __forceinline__ uint32_t ld_b32(const __nv_bfloat16* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kMmaWarps * 32)
router_logits_mma_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                         const float* __restrict__ bias, const __nv_bfloat16* __restrict__ gate_w, int T,
                         int H, int E, float score_scale, float* __restrict__ logits,
                         float* __restrict__ gate_logit) {
  griddep_launch();
  griddep_wait();
  __shared__ float part[kMmaWarps][16][32];  // per-warp partial [token][expert]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tok0 = blockIdx.x * kMmaTok;
  const int e0 = blockIdx.y * kMmaExp;
  const int rows = E + (gate_w != nullptr ? 1 : 0);
  const __nv_bfloat16* xa = x + (int64_t)min(tok0 + g, T - 1) * H + 2 * t;
  const __nv_bfloat16* xb = x + (int64_t)min(tok0 + g + 8, T - 1) * H + 2 * t;
  const __nv_bfloat16* wr[4];
  bool wv[4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int e = e0 + nt * 8 + g;
    wv[nt] = e < rows;
    wr[nt] = wv[nt] ? (e < E ? w + (int64_t)e * H : gate_w) + 2 * t : xa;  // xa: any valid address
  }
  float acc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[nt][q] = 0.f;
#pragma unroll 8
  for (int k0 = warp * 16; k0 < H; k0 += 16 * kMmaWarps) {
    const uint32_t a0 = ld_b32(xa + k0), a1 = ld_b32(xb + k0);
    const uint32_t a2 = ld_b32(xa + k0 + 8), a3 = ld_b32(xb + k0 + 8);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const uint32_t b0 = wv[nt] ? ld_b32(wr[nt] + k0) : 0u;
      const uint32_t b1 = wv[nt] ? ld_b32(wr[nt] + k0 + 8) : 0u;
      mma_bf16_16816(acc[nt], a0, a1, a2, a3, b0, b1);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int q = 0; q < 4; ++q) part[warp][g + (q >= 2 ? 8 : 0)][nt * 8 + 2 * t + (q & 1)] = acc[nt][q];
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * 32; i += kMmaWarps * 32) {
    const int tt = i >> 5, ee = i & 31;
    const int tok = tok0 + tt, e = e0 + ee;
    if (tok >= T || e >= rows) continue;
    float v = 0.f;
#pragma unroll
    for (int ww = 0; ww < kMmaWarps; ++ww) v += part[ww][tt][ee];
    if (e < E) {
      if (bias != nullptr) v += bias[e];
      logits[(int64_t)tok * E + e] = v * score_scale;
    } else {
      gate_logit[tok] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Fused bf16 router: logits + top-k + softmax-over-k + renormalisation + shared
// gate in ONE launch. A cluster of G CTAs (grid.y, G <= 8) owns 16 tokens; CTA r
// of the cluster computes expert rows [r * slice, (r + 1) * slice) in passes of
// 64 rows (8 mma n-tiles), and rank 0 gathers the logit slices through
// distributed shared memory and runs the top-k. G grows at decode sizes so
// that more SMs share the weight stream. kFusedWarps warps split K in 32-wide chunks; within a
// chunk lane (g, t) loads 8 consecutive elements [8t, 8t + 8) of its token rows
// g and g + 8 and of expert row g of each n-tile (16-byte loads) and feeds
// elements 0-3 to one m16n8k16 MMA and 4-7 to a second: both operands see the
// same permutation of K, so each MMA still forms sum_k x[k] w[k]. Products of
// bf16 are exact in fp32; the per-warp partials are summed through shared
// memory in a fixed order (deterministic).
// ---------------------------------------------------------------------------
constexpr int kFusedPass = 64;  // expert rows per pass
constexpr int kFusedMaxRows = 257;

// One warp, one token: K rounds of a warp argmax (ties to the lower expert id);
// lane k keeps slot k in registers, then the softmax over the k selected and
// the renormalisation run lane-parallel. Returns nothing; lanes < K write.
__device__ __forceinline__ void topk_warp(const float* lr, int E, int K, int renorm, float eps, int64_t t,
                                          float* probs, int64_t* idx_out, float* w_out) {
  const int lane = threadIdx.x & 31;
  float mine[8];  // this lane's experts lane + 32 * j (E <= 256)
#pragma unroll
  for (int j = 0; j < 8; ++j) mine[j] = (lane + 32 * j < E) ? lr[lane + 32 * j] : -INFINITY;
  uint32_t taken = 0;
  float my_v = -INFINITY, top = 0.f;
  int my_i = 0;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !(taken & (1u << j)) && (bi == 0x7fffffff || mine[j] > best)) {
        best = mine[j];
        bi = e;
      }
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
    if (k == 0) top = best;
    if (lane == k) {
      my_v = best;
      my_i = bi;
    }
  }
  // softmax over the K selected (max = slot 0), then renormalise by max(sum, eps)
  float p = lane < K ? expf(my_v - top) : 0.f;
  float s = p;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  p = p / s;
  float psum = p;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
  // renorm == 2: the selected experts' probabilities under the softmax over ALL E logits,
  // not renormalised (Hugging Face Qwen2-MoE with norm_topk_prob = false)
  float full = 0.f;
  if (renorm == 2) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane + 32 * j < E) full += expf(mine[j] - top);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) full += __shfl_xor_sync(0xffffffffu, full, off);
  }
  if (lane < K) {
    const int64_t o = t * K + lane;
    idx_out[o] = my_i;
    if (probs != nullptr) probs[o] = p;
    w_out[o] = renorm == 2 ? expf(my_v - top) / full : (K == 1) ? 1.0f : (renorm ? p / fmaxf(psum, eps) : p);
  }
}

// kFusedWarps = 16 at decode sizes (one CTA per SM, the most warps per token tile); 8 when the
// token tiles alone cover the SMs (two CTAs per SM: the T = 4096 grid resident in one wave).
template <int kFusedWarps>
__global__ void __launch_bounds__(kFusedWarps * 32, 16 / kFusedWarps)
router_fused_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                    const float* __restrict__ bias, const __nv_bfloat16* __restrict__ gate_w, int T, int H,
                    int E, int K, float score_scale, int renorm, float eps, float* __restrict__ logits,
                    float* __restrict__ probs, int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                    float* __restrict__ shared_gate) {
  extern __shared__ float fsm[];
  float* part = fsm;                                   // [kFusedWarps][16][kFusedPass]
  float* lg = part + kFusedWarps * 16 * kFusedPass;    // [16][kFusedMaxRows]
  cg::cluster_group cluster = cg::this_cluster();
  const int G = (int)cluster.num_blocks();            // CTAs sharing this token tile
  const int rank = (int)cluster.block_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tok0 = blockIdx.x * 16;
  const int rows = E + (gate_w != nullptr ? 1 : 0);
  const int slice = ((rows + G * 8 - 1) / (G * 8)) * 8;  // expert rows per CTA (whole n-tiles)
  const int e_lo = min(rows, rank * slice), e_hi = min(rows, e_lo + slice);
  const __nv_bfloat16* xa = x + (int64_t)min(tok0 + g, T - 1) * H + 8 * t;
  const __nv_bfloat16* xb = x + (int64_t)min(tok0 + g + 8, T - 1) * H + 8 * t;
  griddep_launch();
  griddep_wait();
  for (int e0 = e_lo; e0 < e_hi; e0 += kFusedPass) {
    const int nts = min(8, (e_hi - e0 + 7) / 8);  // live n-tiles this pass (CTA-uniform)
    const __nv_bfloat16* wr[8];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int e = e0 + nt * 8 + g;
      wr[nt] = e < e_hi ? (e < E ? w + (int64_t)e * H : gate_w) + 8 * t : xa;  // xa: any valid row
    }
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[nt][q] = 0.f;
#pragma unroll 2
    for (int k0 = warp * 32; k0 < H; k0 += 32 * kFusedWarps) {
      const uint4 va = *reinterpret_cast<const uint4*>(xa + k0);
      const uint4 vb = *reinterpret_cast<const uint4*>(xb + k0);
      uint4 bw[8];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
        bw[nt] = nt < nts ? *reinterpret_cast<const uint4*>(wr[nt] + k0) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        if (nt < nts) {
          mma_bf16_16816(acc[nt], va.x, vb.x, va.y, vb.y, bw[nt].x, bw[nt].y);
          mma_bf16_16816(acc[nt], va.z, vb.z, va.w, vb.w, bw[nt].z, bw[nt].w);
        }
      }
    }
    float* pw = part + warp * 16 * kFusedPass;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      if (nt < nts) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          pw[(g + (q >= 2 ? 8 : 0)) * kFusedPass + nt * 8 + 2 * t + (q & 1)] = acc[nt][q];
      }
    __syncthreads();
    const int width = nts * 8;
    for (int i = threadIdx.x; i < 16 * width; i += kFusedWarps * 32) {
      const int tt = i / width, ee = i % width;
      const int tok = tok0 + tt, e = e0 + ee;
      if (tok >= T || e >= e_hi) continue;
      float v = 0.f;
#pragma unroll
      for (int ww = 0; ww < kFusedWarps; ++ww) v += part[(ww * 16 + tt) * kFusedPass + ee];
      if (e < E) {
        if (bias != nullptr) v += bias[e];
        v *= score_scale;
        logits[(int64_t)tok * E + e] = v;
      }
      lg[tt * kFusedMaxRows + e] = v;
    }
    __syncthreads();
  }
  if (G > 1) {
    // rank 0 collects the other CTAs' logit slices through distributed shared memory
    cluster.sync();
    if (rank == 0) {
      for (int r = 1; r < G; ++r) {
        const int lo = min(rows, r * slice), hi = min(rows, lo + slice);
        const float* rlg = cluster.map_shared_rank(lg, r);
        for (int i = threadIdx.x; i < 16 * (hi - lo); i += kFusedWarps * 32) {
          const int tt = i / (hi - lo), e = lo + i % (hi - lo);
          lg[tt * kFusedMaxRows + e] = rlg[tt * kFusedMaxRows + e];
        }
      }
    }
    cluster.sync();  // the other CTAs stay resident until rank 0 has read them
    if (rank != 0) return;
  }
  // one warp per token: top-k, softmax over k, renormalisation, sigmoid shared gate
  for (int tt = warp; tt < 16; tt += kFusedWarps) {
    const int tok = tok0 + tt;
    if (tok < T) {
      const float* lr = lg + tt * kFusedMaxRows;
      topk_warp(lr, E, K, renorm, eps, tok, probs, idx_out, w_out);
      if (lane == 0 && gate_w != nullptr) shared_gate[tok] = 1.0f / (1.0f + expf(-lr[E]));
    }
  }
}

constexpr size_t fused_smem(int warps) { return (size_t)(warps * 16 * kFusedPass + 16 * kFusedMaxRows) * sizeof(float); }

// Top-k + softmax over the k selected + renormalisation: one warp per token.
__global__ void __launch_bounds__(kRouterThreads)
router_topk_kernel(const float* __restrict__ logits, int T, int E, int K, int renorm, float eps,
                   float* __restrict__ probs, int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                   float* __restrict__ shared_gate) {
  griddep_launch();
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (kRouterThreads / 32) + warp;
  if (t >= T) return;
  if (shared_gate != nullptr && lane == 0) shared_gate[t] = 1.0f / (1.0f + expf(-shared_gate[t]));
  topk_warp(logits + (int64_t)t * E, E, K, renorm, eps, t, probs, idx_out, w_out);
}


// ---------------------------------------------------------------------------
// Decode-sized batches (T * K <= 256, E <= 256, bf16): router AND dispatch in ONE
// launch. CTA e < E computes expert e's logits for every token (its 2-byte weight row
// is read once, each of the 256 threads holding 8 elements of it); CTA E computes the
// shared gate's logit. The last CTA to finish (a ticket counter in device memory,
// reset by that CTA for the next launch) runs top-k / softmax / renormalisation per
// token (one warp per token) and the stable counting sort of the T * K assignments:
// dest[i] = offsets[e_i] + #{j < i : e_j == e_i}, the reference counting scatter
// (DWDP/dispatcher/kernels/reference.py:163-257). With one expert row per CTA the
// router's weight stream spreads over E SMs instead of one cluster.
// ---------------------------------------------------------------------------
constexpr int kRdThreads = 256;
constexpr int kRdMaxN = 256;  // assignments

__global__ void __launch_bounds__(kRdThreads)
route_dispatch_small_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                            const float* __restrict__ bias, const __nv_bfloat16* __restrict__ gate_w, int T,
                            int H, int E, int K, float score_scale, int renorm, float eps,
                            float* __restrict__ logits, float* __restrict__ gate_logit, float* __restrict__ probs,
                            int64_t* __restrict__ idx_out, float* __restrict__ w_out,
                            float* __restrict__ shared_gate, int64_t* __restrict__ counts,
                            int64_t* __restrict__ offsets, int64_t* __restrict__ perm, int64_t* __restrict__ inv,
                            int64_t* __restrict__ ids, int64_t* __restrict__ tok, float* __restrict__ packed_w,
                            int* __restrict__ ticket, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  __shared__ float s_part[kRdThreads / 32][64];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = blockIdx.x;  // expert row, or E for the shared gate
  const __nv_bfloat16* wr = row < E ? w + (int64_t)row * H : gate_w;
  // ---- 1. logits of this row for every token (tokens in chunks of 32)
  for (int t0 = 0; t0 < T; t0 += 32) {
    const int nt = min(32, T - t0);
    float part[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) part[t] = 0.f;
    for (int c = tid * 8; c < H; c += kRdThreads * 8) {
      float wv[8];
      load8(wr + c, wv);
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        if (t < nt) {
          float xv[8];
          load8(x + (int64_t)(t0 + t) * H + c, xv);
          float s = part[t];
#pragma unroll
          for (int q = 0; q < 8; ++q) s = fmaf(xv[q], wv[q], s);
          part[t] = s;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      if (t < nt) {
        float v = part[t];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) s_part[warp][t] = v;
      }
    }
    __syncthreads();
    if (tid < nt) {
      float v = 0.f;
#pragma unroll
      for (int ww = 0; ww < kRdThreads / 32; ++ww) v += s_part[ww][tid];
      if (row < E) {
        if (bias != nullptr) v += bias[row];
        logits[(int64_t)(t0 + tid) * E + row] = v * score_scale;
      } else {
        gate_logit[t0 + tid] = v;
      }
    }
    __syncthreads();
  }
  // ---- 2. the last CTA to finish routes and dispatches
  __threadfence();
  if (tid == 0) {
    const int done = atomicAdd(ticket, 1);
    s_last = done == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) *ticket = 0;  // ready for the next launch
  // top-k / softmax / renormalisation, one warp per token, on the logits the other CTAs wrote
  __shared__ float s_lg[kRdThreads / 32][256];
  for (int t = warp; t < T; t += kRdThreads / 32) {
    for (int e = lane; e < E; e += 32) s_lg[warp][e] = __ldcg(logits + (int64_t)t * E + e);
    __syncwarp();
    topk_warp(s_lg[warp], E, K, renorm, eps, t, probs, idx_out, w_out);
    if (lane == 0 && gate_w != nullptr) shared_gate[t] = 1.0f / (1.0f + expf(-__ldcg(gate_logit + t)));
    __syncwarp();
  }
  __syncthreads();
  // stable counting sort of the N = T * K assignments (token-major order i = t * K + k)
  __shared__ int s_e[kRdMaxN];
  __shared__ int s_cnt[256];
  __shared__ int s_off[257];
  const int N = T * K;
  for (int e = tid; e < E; e += kRdThreads) s_cnt[e] = 0;
  __syncthreads();
  int my_e = -1;
  if (tid < N) {
    my_e = (int)__ldcg(idx_out + tid);
    s_e[tid] = my_e;
    if (my_e >= 0 && my_e < E) atomicAdd(&s_cnt[my_e], 1);
    else record_error(st, DWDP_ERR_DEVICE_BOUNDS, 102, tid);
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan over E <= 256 experts: 8 per lane, then across lanes
    int loc[8], sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane * 8 + j;
      loc[j] = e < E ? s_cnt[e] : 0;
      sum += loc[j];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - sum;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane * 8 + j;
      if (e < E) s_off[e] = run;
      run += loc[j];
    }
    if (lane == 31) s_off[E] = incl;
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRdThreads) {
    counts[e] = s_cnt[e];
    offsets[e] = s_off[e];
  }
  if (tid == 0) offsets[E] = s_off[E];
  if (tid < N && my_e >= 0 && my_e < E) {
    int rank = 0;
    for (int j = 0; j < tid; ++j) rank += s_e[j] == my_e;
    const int d = s_off[my_e] + rank;
    perm[d] = tid;
    inv[tid] = d;
    ids[d] = my_e;
    tok[d] = tid / K;
    packed_w[d] = __ldcg(w_out + tid);
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
  if (H % 8 != 0 || logits == nullptr) return DWDP_ERR_INVALID_ARGUMENT;
  const int rows = E + (shared_gate_weight != nullptr ? 1 : 0);
  int tok = 16;
  const size_t xsz = hidden_dtype == DWDP_DTYPE_F32 ? 4 : 2;
  while (tok > 2 && ((size_t)tok * H * xsz > 96 * 1024 || tok / 2 >= T)) tok /= 2;
  if ((size_t)tok * H * xsz > 200 * 1024) return DWDP_ERR_UNSUPPORTED;
  const size_t smem = (size_t)tok * H * xsz;
  const dim3 grid((unsigned)((T + tok - 1) / tok), (unsigned)((rows + 7) / 8));
#define DWDP_LAUNCH_LOGITS(TX, TW, TOKN)                                                              \
  do {                                                                                                \
    auto kfn = router_logits_kernel<TX, TW, TOKN>;                                                    \
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=         \
        cudaSuccess)                                                                                  \
      return DWDP_ERR_CUDA;                                                                           \
    if (launch_chained(kfn, grid, dim3(kRouterThreads), smem, stream, 1u, (const TX*)hidden,          \
                       (const TW*)weight, bias, (const TW*)shared_gate_weight, (int)T, H, E,          \
                       score_scale, logits, shared_gate) != cudaSuccess)                              \
      return DWDP_ERR_CUDA;                                                                           \
  } while (0)
#define DWDP_LOGITS_TOK(TX, TW)                          \
  do {                                                   \
    if (tok == 16) DWDP_LAUNCH_LOGITS(TX, TW, 16);       \
    else if (tok == 8) DWDP_LAUNCH_LOGITS(TX, TW, 8);    \
    else if (tok == 4) DWDP_LAUNCH_LOGITS(TX, TW, 4);    \
    else DWDP_LAUNCH_LOGITS(TX, TW, 2);                  \
  } while (0)
  if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_BF16 && H % 32 == 0 && E <= 256 &&
      K <= 16) {
    // expert slices per token tile: enough CTAs to cover the SMs at decode sizes
    const int64_t tiles = (T + 15) / 16;
    const bool wide_grid = tiles >= 148;  // prefill: 8-warp CTAs, two per SM
    auto kfn = wide_grid ? router_fused_kernel<8> : router_fused_kernel<16>;
    const size_t smem = fused_smem(wide_grid ? 8 : 16);
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return DWDP_ERR_CUDA;
    int G = 1;
    while (G < 8 && tiles * G < 148 && G * 8 < rows) G *= 2;
    if (const char* v = getenv("DWDP_ROUTER_G")) {  // tuning override: cluster size 1, 2, 4 or 8
      const int g = atoi(v);
      if (g == 1 || g == 2 || g == 4 || g == 8) G = g;
    }
    if (launch_chained(kfn, dim3((unsigned)tiles, (unsigned)G, 1), dim3((wide_grid ? 8 : 16) * 32, 1, 1),
                       smem, stream, (unsigned)G, (const __nv_bfloat16*)hidden,
                       (const __nv_bfloat16*)weight, bias, (const __nv_bfloat16*)shared_gate_weight, (int)T, H, E, K,
                       score_scale, renorm, eps, logits, probs, idx, topk_w, shared_gate) != cudaSuccess)
      return DWDP_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
  }
  if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_BF16 && H % 16 == 0) {
    const dim3 mgrid((unsigned)((T + kMmaTok - 1) / kMmaTok), (unsigned)((rows + kMmaExp - 1) / kMmaExp));
    if (launch_chained(router_logits_mma_kernel, mgrid, dim3(kMmaWarps * 32), 0, stream, 1u,
                       (const __nv_bfloat16*)hidden, (const __nv_bfloat16*)weight, bias,
                       (const __nv_bfloat16*)shared_gate_weight, (int)T, H, E, score_scale, logits,
                       shared_gate) != cudaSuccess)
      return DWDP_ERR_CUDA;
  } else if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_BF16)
    DWDP_LOGITS_TOK(__nv_bfloat16, __nv_bfloat16);
  else if (hidden_dtype == DWDP_DTYPE_BF16 && weight_dtype == DWDP_DTYPE_F32)
    DWDP_LOGITS_TOK(__nv_bfloat16, float);
  else if (hidden_dtype == DWDP_DTYPE_F32 && weight_dtype == DWDP_DTYPE_F32)
    DWDP_LOGITS_TOK(float, float);
  else if (hidden_dtype == DWDP_DTYPE_F32 && weight_dtype == DWDP_DTYPE_BF16)
    DWDP_LOGITS_TOK(float, __nv_bfloat16);
  else
    return DWDP_ERR_UNSUPPORTED;
#undef DWDP_LOGITS_TOK
#undef DWDP_LAUNCH_LOGITS
  const unsigned tk_grid = (unsigned)((T + 7) / 8);
  if (launch_chained(router_topk_kernel, dim3(tk_grid), dim3(kRouterThreads), 0, stream, 1u, (const float*)logits,
                     (int)T, E, K, renorm, eps, probs, idx, topk_w,
                     shared_gate_weight ? shared_gate : (float*)nullptr) != cudaSuccess)
    return DWDP_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

// Router + dispatch in one launch for decode-sized batches (see route_dispatch_small_kernel).
// Returns DWDP_ERR_UNSUPPORTED outside its range (the caller then launches the two stages).
extern "C" int dwdp_route_dispatch_small_launch(const void* hidden, const void* weight, const float* bias,
                                                const void* shared_gate_weight, int64_t T, int H, int E, int K,
                                                float score_scale, int renorm, float eps, float* logits,
                                                float* gate_logit, float* probs, int64_t* idx, float* topk_w,
                                                float* shared_gate, int64_t* counts, int64_t* offsets,
                                                int64_t* perm, int64_t* inv, int64_t* ids, int64_t* tok,
                                                float* packed_w, int* ticket, int* status, cudaStream_t stream) {
  if (T <= 0 || T * K > kRdMaxN || E > 256 || K > 16 || K > E || H % 8 != 0) return DWDP_ERR_UNSUPPORTED;
  if (shared_gate_weight != nullptr && (gate_logit == nullptr || shared_gate == nullptr))
    return DWDP_ERR_INVALID_ARGUMENT;
  const int rows = E + (shared_gate_weight != nullptr ? 1 : 0);
  return launch_chained(route_dispatch_small_kernel, dim3((unsigned)rows), dim3(kRdThreads), 0, stream, 1u,
                        (const __nv_bfloat16*)hidden, (const __nv_bfloat16*)weight, bias,
                        (const __nv_bfloat16*)shared_gate_weight, (int)T, H, E, K, score_scale, renorm, eps, logits,
                        gate_logit, probs, idx, topk_w, shared_gate, counts, offsets, perm, inv, ids, tok, packed_w,
                        ticket, reinterpret_cast<DeviceStatus*>(status)) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

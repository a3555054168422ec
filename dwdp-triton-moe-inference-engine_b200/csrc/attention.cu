// Decode-step attention pieces for the full Qwen1.5-MoE decode step (the model
// around the MoE layers): fused residual-add + RMSNorm, RoPE + paged-KV append,
// and paged decode attention (split over the context, then combined).
//
// Follows the reference's decode-step shape (DWDP/adapters/qwen15_moe.py, the
// HF Qwen2-MoE block it wraps, and DWDP/runtime/paged_attention.py:20-76 for
// the block-table cache: [num_blocks, block_size, heads, head_dim]); attention
// itself is "any correct implementation" for this row.
#include "common.cuh"

namespace dwdp {

// ---------------------------------------------------------------------------
// out = rmsnorm(x + delta) * w ; x <- x + delta (the residual stream) when delta given.
// One CTA per row, fp32 sums.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(__nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ delta,
                                                          const __nv_bfloat16* __restrict__ w, int H, float eps,
                                                          __nv_bfloat16* __restrict__ out) {
  griddep_launch();
  griddep_wait();
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  __nv_bfloat16* xr = x + (size_t)row * H;
  const __nv_bfloat16* dr = delta != nullptr ? delta + (size_t)row * H : nullptr;
  float ss = 0.f;
  for (int c = tid * 8; c < H; c += 256 * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    __nv_bfloat162* b = reinterpret_cast<__nv_bfloat162*>(&v);
    if (dr != nullptr) {
      const uint4 d = *reinterpret_cast<const uint4*>(dr + c);
      const __nv_bfloat162* db = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a = __bfloat1622float2(b[q]), e = __bfloat1622float2(db[q]);
        b[q] = __floats2bfloat162_rn(a.x + e.x, a.y + e.y);
      }
      *reinterpret_cast<uint4*>(xr + c) = v;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = __bfloat1622float2(b[q]);
      ss += a.x * a.x + a.y * a.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)H + eps);
  for (int c = tid * 8; c < H; c += 256 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* wb = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = __bfloat1622float2(b[q]), ww = __bfloat1622float2(wb[q]);
      ob[q] = __floats2bfloat162_rn(a.x * r * ww.x, a.y * r * ww.y);
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * H + c) = o;
  }
}

// ---------------------------------------------------------------------------
// qkv [B, 3, NH, D] (+ bias) -> q [B, NH, D] with rotary embedding; k (rotated) and
// v written at position pos[b] of sequence b's paged cache
// ([num_blocks, block_size, NH, D], block b_t = block_table[b][pos / block_size]).
// Rotary: NeoX layout (pairs d, d + D/2), inv_freq = theta^(-2d/D). One CTA per
// (token, head), D/2 threads.
// ---------------------------------------------------------------------------
__global__ void rope_append_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ bias,
                                   const int32_t* __restrict__ pos, const int32_t* __restrict__ block_table,
                                   int max_blocks, int NH, int D, int block_size, float theta,
                                   __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                   __nv_bfloat16* __restrict__ v_cache, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;  // d < D/2
  const int half = D / 2;
  const int p = pos[b];
  const int blk = block_table[(size_t)b * max_blocks + p / block_size];
  if (blk < 0) {
    if (d == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 400, b);
    return;
  }
  const size_t row = (size_t)b * 3 * NH * D;
  auto ld = [&](int which, int dd) {
    const size_t i = (size_t)which * NH * D + (size_t)h * D + dd;
    float v = __bfloat162float(qkv[row + i]);
    if (bias != nullptr) v += __bfloat162float(bias[i]);
    return v;
  };
  const float inv_freq = powf(theta, -2.0f * (float)d / (float)D);
  float sn, cs;
  sincosf((float)p * inv_freq, &sn, &cs);
  const float q0 = ld(0, d), q1 = ld(0, d + half);
  const float k0 = ld(1, d), k1 = ld(1, d + half);
  __nv_bfloat16* qo = q_out + ((size_t)b * NH + h) * D;
  qo[d] = __float2bfloat16_rn(q0 * cs - q1 * sn);
  qo[d + half] = __float2bfloat16_rn(q1 * cs + q0 * sn);
  const size_t slot = (((size_t)blk * block_size + p % block_size) * NH + h) * D;
  k_cache[slot + d] = __float2bfloat16_rn(k0 * cs - k1 * sn);
  k_cache[slot + d + half] = __float2bfloat16_rn(k1 * cs + k0 * sn);
  v_cache[slot + d] = __float2bfloat16_rn(ld(2, d));
  v_cache[slot + d + half] = __float2bfloat16_rn(ld(2, d + half));
}

// ---------------------------------------------------------------------------
// Paged decode attention, split over the context (flash-decoding): CTA (b, h, s)
// covers positions [s * chunk, min(len, (s + 1) * chunk)) of sequence b with 4
// warps; a warp takes one position at a time (lane l holds dims 4l..4l+3), keeps
// an online softmax (running max m, sum l, accumulator), and the 4 warps merge in
// shared memory. Partials (m, l, acc[D]) go to the workspace; the combine kernel
// rescales them into out[b, h, :]. D = 128.
// ---------------------------------------------------------------------------
constexpr int kAttnWarps = 4;
constexpr int kHeadDim = 128;
constexpr int kPos = 8;

__global__ void __launch_bounds__(kAttnWarps * 32)
paged_decode_attn_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
                         const __nv_bfloat16* __restrict__ v_cache, const int32_t* __restrict__ block_table,
                         const int32_t* __restrict__ seq_lens, int max_blocks, int NH, int block_size, int chunk,
                         float scale, float* __restrict__ part_ml, float* __restrict__ part_acc) {
  griddep_launch();
  griddep_wait();
  __shared__ float s_m[kAttnWarps], s_l[kAttnWarps];
  __shared__ float s_acc[kAttnWarps][kHeadDim];
  const int b = blockIdx.x, h = blockIdx.y, sp = blockIdx.z, S = gridDim.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_lens[b];
  const int p0 = sp * chunk, p1 = min(len, p0 + chunk);
  float qv[4];
  {
    const uint2 u = *reinterpret_cast<const uint2*>(q + ((size_t)b * NH + h) * kHeadDim + 4 * lane);
    const __nv_bfloat162* qb = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(qb[0]), c = __bfloat1622float2(qb[1]);
    qv[0] = a.x * scale; qv[1] = a.y * scale; qv[2] = c.x * scale; qv[3] = c.y * scale;
  }
  // Each warp takes groups of kPos consecutive positions (group g at p0 + (g * W + warp) * kPos):
  // all K/V rows of a group are loaded before any arithmetic, so a warp keeps
  // 2 * kPos 256-byte rows in flight.
  float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int g0 = p0 + warp * kPos; g0 < p1; g0 += kAttnWarps * kPos) {
    uint2 ku[kPos], vu[kPos];
#pragma unroll
    for (int j = 0; j < kPos; ++j) {
      const int p = g0 + j;
      if (p < p1) {
        const int blk = block_table[(size_t)b * max_blocks + p / block_size];
        const size_t off = (((size_t)blk * block_size + p % block_size) * NH + h) * kHeadDim + 4 * lane;
        ku[j] = __ldg(reinterpret_cast<const uint2*>(k_cache + off));
        vu[j] = __ldg(reinterpret_cast<const uint2*>(v_cache + off));
      } else {
        ku[j] = make_uint2(0u, 0u);
        vu[j] = make_uint2(0u, 0u);
      }
    }
    float sc[kPos];
#pragma unroll
    for (int j = 0; j < kPos; ++j) {
      const __nv_bfloat162* kb = reinterpret_cast<const __nv_bfloat162*>(&ku[j]);
      const float2 k0 = __bfloat1622float2(kb[0]), k1 = __bfloat1622float2(kb[1]);
      sc[j] = qv[0] * k0.x + qv[1] * k0.y + qv[2] * k1.x + qv[3] * k1.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int j = 0; j < kPos; ++j) sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], o);
    }
    float mn = m;
#pragma unroll
    for (int j = 0; j < kPos; ++j)
      if (g0 + j < p1) mn = fmaxf(mn, sc[j]);
    const float corr = expf(m - mn);
    l *= corr;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] *= corr;
#pragma unroll
    for (int j = 0; j < kPos; ++j) {
      const float pe = g0 + j < p1 ? expf(sc[j] - mn) : 0.f;
      const __nv_bfloat162* vb = reinterpret_cast<const __nv_bfloat162*>(&vu[j]);
      const float2 v0 = __bfloat1622float2(vb[0]), v1 = __bfloat1622float2(vb[1]);
      l += pe;
      acc[0] += pe * v0.x;
      acc[1] += pe * v0.y;
      acc[2] += pe * v1.x;
      acc[3] += pe * v1.y;
    }
    m = mn;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s_acc[warp][4 * lane + i] = acc[i];
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = s_m[w] == -INFINITY ? 0.f : expf(s_m[w] - M);
      L += s_l[w] * f;
#pragma unroll
      for (int i = 0; i < 4; ++i) A[i] += s_acc[w][4 * lane + i] * f;
    }
    const size_t pi = ((size_t)b * NH + h) * S + sp;
    if (lane == 0) {
      part_ml[2 * pi] = M;
      part_ml[2 * pi + 1] = L;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) part_acc[pi * kHeadDim + 4 * lane + i] = A[i];
  }
}

// out[b, h, :] = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s ; one warp per (b, h).
__global__ void attn_combine_kernel(const float* __restrict__ part_ml, const float* __restrict__ part_acc, int S,
                                    int BH, __nv_bfloat16* __restrict__ out) {
  griddep_launch();
  griddep_wait();
  const int bh = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (bh >= BH) return;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, part_ml[2 * ((size_t)bh * S + s)]);
  float L = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < S; ++s) {
    const size_t pi = (size_t)bh * S + s;
    const float ms = part_ml[2 * pi];
    const float f = ms == -INFINITY ? 0.f : expf(ms - M);
    L += part_ml[2 * pi + 1] * f;
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] += part_acc[pi * kHeadDim + 4 * lane + i] * f;
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) out[(size_t)bh * kHeadDim + 4 * lane + i] = __float2bfloat16_rn(A[i] * inv);
}

}  // namespace dwdp

using namespace dwdp;

extern "C" int dwdp_add_rmsnorm_launch(void* x, const void* delta, const void* w, int64_t rows, int H, float eps,
                                       void* out, cudaStream_t stream) {
  if (rows <= 0) return DWDP_OK;
  if (H % 8 || H > 256 * 8 * 64) return DWDP_ERR_INVALID_ARGUMENT;
  return launch_chained(add_rmsnorm_kernel, dim3((unsigned)rows), dim3(256), 0, stream, 1u, (__nv_bfloat16*)x,
                        (const __nv_bfloat16*)delta, (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)out) ==
                 cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

extern "C" int dwdp_rope_append_launch(const void* qkv, const void* bias, const int32_t* pos,
                                       const int32_t* block_table, int B, int max_blocks, int NH, int D,
                                       int block_size, float theta, void* q_out, void* k_cache, void* v_cache,
                                       int* status, cudaStream_t stream) {
  if (B <= 0) return DWDP_OK;
  if (D % 2 || D > 1024 || block_size <= 0) return DWDP_ERR_INVALID_ARGUMENT;
  return launch_chained(rope_append_kernel, dim3((unsigned)B, (unsigned)NH), dim3(D / 2), 0, stream, 1u,
                        (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)bias, pos, block_table, max_blocks, NH, D,
                        block_size, theta, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache,
                        reinterpret_cast<DeviceStatus*>(status)) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

extern "C" size_t dwdp_paged_attention_workspace_bytes_impl(int B, int NH, int splits) {
  const size_t n = (size_t)B * NH * splits;
  return n * 2 * sizeof(float) + n * kHeadDim * sizeof(float) + 256;
}

// splits: context chunks per (sequence, head); chunk = ceil(max_len / splits) positions.
extern "C" int dwdp_paged_attention_launch(const void* q, const void* k_cache, const void* v_cache,
                                           const int32_t* block_table, const int32_t* seq_lens, int B,
                                           int max_blocks, int NH, int D, int block_size, int max_len, int splits,
                                           float scale, void* workspace, void* out, cudaStream_t stream) {
  if (B <= 0) return DWDP_OK;
  if (D != kHeadDim || splits <= 0 || max_len <= 0) return DWDP_ERR_UNSUPPORTED;
  float* part_ml = reinterpret_cast<float*>(workspace);
  float* part_acc = part_ml + (size_t)B * NH * splits * 2;
  const int chunk = (max_len + splits - 1) / splits;
  if (launch_chained(paged_decode_attn_kernel, dim3((unsigned)B, (unsigned)NH, (unsigned)splits),
                     dim3(kAttnWarps * 32), 0, stream, 1u, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k_cache,
                     (const __nv_bfloat16*)v_cache, block_table, seq_lens, max_blocks, NH, block_size, chunk, scale,
                     part_ml, part_acc) != cudaSuccess)
    return DWDP_ERR_CUDA;
  const int BH = B * NH;
  return launch_chained(attn_combine_kernel, dim3((unsigned)((BH + 7) / 8)), dim3(256), 0, stream, 1u,
                        (const float*)part_ml, (const float*)part_acc, splits, BH, (__nv_bfloat16*)out) ==
                 cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

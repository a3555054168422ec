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
                                   int max_blocks, int num_blocks, int NH, int D, int block_size, float theta,
                                   __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                   __nv_bfloat16* __restrict__ v_cache, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;  // d < D/2
  const int half = D / 2;
  const int p = pos[b];
  // the position must lie inside the block table and its block inside the cache
  const int blk = (p >= 0 && p < max_blocks * block_size) ? block_table[(size_t)b * max_blocks + p / block_size] : -1;
  if (blk < 0 || blk >= num_blocks) {
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
                         const int32_t* __restrict__ seq_lens, int max_blocks, int num_blocks, int NH,
                         int block_size, int chunk, float scale, float* __restrict__ part_ml,
                         float* __restrict__ part_acc, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  __shared__ float s_m[kAttnWarps], s_l[kAttnWarps];
  __shared__ float s_acc[kAttnWarps][kHeadDim];
  const int b = blockIdx.x, h = blockIdx.y, sp = blockIdx.z, S = gridDim.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = min(seq_lens[b], max_blocks * block_size);  // never past the block table
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
    bool use[kPos];  // inside the chunk and in a valid block (a bad block id is recorded and skipped)
#pragma unroll
    for (int j = 0; j < kPos; ++j) {
      const int p = g0 + j;
      use[j] = false;
      ku[j] = make_uint2(0u, 0u);
      vu[j] = make_uint2(0u, 0u);
      if (p < p1) {
        const int blk = block_table[(size_t)b * max_blocks + p / block_size];
        if (blk < 0 || blk >= num_blocks) {
          if (lane == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 402, b);
        } else {
          const size_t off = (((size_t)blk * block_size + p % block_size) * NH + h) * kHeadDim + 4 * lane;
          ku[j] = __ldg(reinterpret_cast<const uint2*>(k_cache + off));
          vu[j] = __ldg(reinterpret_cast<const uint2*>(v_cache + off));
          use[j] = true;
        }
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
      if (use[j]) mn = fmaxf(mn, sc[j]);
    const float corr = mn == -INFINITY ? 1.f : expf(m - mn);
    l *= corr;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] *= corr;
#pragma unroll
    for (int j = 0; j < kPos; ++j) {
      const float pe = use[j] ? expf(sc[j] - mn) : 0.f;
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

// ---------------------------------------------------------------------------
// Paged decode attention, bulk-copy pipeline. In the cache layout
// [blocks, block_size, NH, D] one position's K (or V) for ALL heads is one
// contiguous NH*D*2-byte row, and kStagePos consecutive positions of one block are
// one contiguous run. CTA (split s, sequence b) covers positions
// [s * chunk, min(len, (s + 1) * chunk)) for every head: warp 8 (producer) streams
// K and V runs into a kStages-deep shared-memory ring with cp.async.bulk (mbarrier
// transaction counts); warps 0..7 (consumers) each own HPW heads (NH = 8 * HPW):
// lane l holds dims 4l..4l+3, a 256-byte head row is one conflict-free shared load
// per warp, and the online softmax state (m, l, acc) stays in registers. Partials
// (m, l, acc[D]) per (b, h, s) go to the workspace for attn_combine_kernel.
// Waits are bounded: a timeout records DWDP_ERR_DEVICE_TIMEOUT and the CTA returns
// after the producer has waited (again bounded) for its copies in flight.
// ---------------------------------------------------------------------------
constexpr int kStagePos = 4;
constexpr int kStages = 3;
constexpr int kConsumerWarps = 8;

template <int HPW>
__global__ void __launch_bounds__((kConsumerWarps + 1) * 32)
paged_attn_bulk_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
                       const __nv_bfloat16* __restrict__ v_cache, const int32_t* __restrict__ block_table,
                       const int32_t* __restrict__ seq_lens, int max_blocks, int num_blocks, int block_size,
                       int chunk, float scale, float* __restrict__ part_ml, float* __restrict__ part_acc,
                       DeviceStatus* st) {
  constexpr int NH = kConsumerWarps * HPW;
  constexpr uint32_t kRow = NH * kHeadDim * 2;             // bytes of one position, all heads
  constexpr uint32_t kRun = kStagePos * kRow;              // bytes of one stage of K (or V)
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* kbuf = smem;                                    // [kStages][kRun]
  uint8_t* vbuf = smem + kStages * kRun;                   // [kStages][kRun]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kRun);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  int* valid = const_cast<int*>(abort_flag) + 1;           // [kStages]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sp = blockIdx.x, S = gridDim.x, b = blockIdx.y;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  griddep_launch();
  griddep_wait();
  const int len = min(seq_lens[b], max_blocks * block_size);  // never past the block table
  const int p0 = sp * chunk, p1 = min(len, p0 + chunk);
  const int nst = p1 > p0 ? (p1 - p0 + kStagePos - 1) / kStagePos : 0;

  if (warp == kConsumerWarps) {
    // ---------------- producer
    if (lane == 0) {
      int i = 0;
      for (; i < nst; ++i) {
        const int slot = i % kStages;
        if (i >= kStages && !mbar_wait(&empty[slot], ((i / kStages) - 1) & 1, abort_flag, st, 410)) break;
        const int p = p0 + i * kStagePos;
        const int blk = block_table[(size_t)b * max_blocks + p / block_size];
        if (blk < 0 || blk >= num_blocks) {
          record_error(st, DWDP_ERR_DEVICE_BOUNDS, 411, b);
          valid[slot] = 0;
          mbar_arrive(&full[slot]);
          continue;
        }
        valid[slot] = 1;
        const size_t off = ((size_t)blk * block_size + p % block_size) * (size_t)(NH * kHeadDim);
        mbar_arrive_expect_tx(&full[slot], 2 * kRun);
        bulk_g2s(kbuf + slot * kRun, k_cache + off, kRun, &full[slot]);
        bulk_g2s(vbuf + slot * kRun, v_cache + off, kRun, &full[slot]);
      }
      // On an abort, let the copies already issued land before the CTA exits.
      if (*abort_flag) {
        for (int j = max(0, i - kStages); j < i; ++j) {
          volatile int dummy = 0;
          mbar_wait(&full[j % kStages], (j / kStages) & 1, &dummy, nullptr, 0);
        }
      }
    }
    return;
  }

  // ---------------- consumers
  float qv[HPW][4], m[HPW], l[HPW], acc[HPW][4];
#pragma unroll
  for (int j = 0; j < HPW; ++j) {
    const int h = warp * HPW + j;
    const uint2 u = *reinterpret_cast<const uint2*>(q + ((size_t)b * NH + h) * kHeadDim + 4 * lane);
    const __nv_bfloat162* qb = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(qb[0]), c = __bfloat1622float2(qb[1]);
    qv[j][0] = a.x * scale; qv[j][1] = a.y * scale; qv[j][2] = c.x * scale; qv[j][3] = c.y * scale;
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
  }
  bool ok = true;
  for (int i = 0; i < nst; ++i) {
    const int slot = i % kStages;
    if (!mbar_wait(&full[slot], (i / kStages) & 1, abort_flag, st, 412)) {
      ok = false;
      break;
    }
    const int npos = min(kStagePos, p1 - (p0 + i * kStagePos));
    if (valid[slot]) {
      const uint8_t* ks = kbuf + slot * kRun;
      const uint8_t* vs = vbuf + slot * kRun;
#pragma unroll
      for (int j = 0; j < HPW; ++j) {
        const int h = warp * HPW + j;
        float sc[kStagePos];
        uint2 vu[kStagePos];
#pragma unroll
        for (int t = 0; t < kStagePos; ++t) {
          const uint2 ku = *reinterpret_cast<const uint2*>(ks + t * kRow + h * kHeadDim * 2 + 8 * lane);
          vu[t] = *reinterpret_cast<const uint2*>(vs + t * kRow + h * kHeadDim * 2 + 8 * lane);
          const __nv_bfloat162* kb = reinterpret_cast<const __nv_bfloat162*>(&ku);
          const float2 k0 = __bfloat1622float2(kb[0]), k1 = __bfloat1622float2(kb[1]);
          sc[t] = qv[j][0] * k0.x + qv[j][1] * k0.y + qv[j][2] * k1.x + qv[j][3] * k1.y;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
          for (int t = 0; t < kStagePos; ++t) sc[t] += __shfl_xor_sync(0xffffffffu, sc[t], o);
        }
        float mn = m[j];
#pragma unroll
        for (int t = 0; t < kStagePos; ++t)
          if (t < npos) mn = fmaxf(mn, sc[t]);
        const float corr = expf(m[j] - mn);
        l[j] *= corr;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[j][c] *= corr;
#pragma unroll
        for (int t = 0; t < kStagePos; ++t) {
          const float pe = t < npos ? expf(sc[t] - mn) : 0.f;
          const __nv_bfloat162* vb = reinterpret_cast<const __nv_bfloat162*>(&vu[t]);
          const float2 v0 = __bfloat1622float2(vb[0]), v1 = __bfloat1622float2(vb[1]);
          l[j] += pe;
          acc[j][0] += pe * v0.x;
          acc[j][1] += pe * v0.y;
          acc[j][2] += pe * v1.x;
          acc[j][3] += pe * v1.y;
        }
        m[j] = mn;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (!ok) return;
#pragma unroll
  for (int j = 0; j < HPW; ++j) {
    const int h = warp * HPW + j;
    const size_t pi = ((size_t)b * NH + h) * S + sp;
    if (lane == 0) {
      part_ml[2 * pi] = m[j];
      part_ml[2 * pi + 1] = l[j];
    }
    *reinterpret_cast<float4*>(part_acc + pi * kHeadDim + 4 * lane) =
        make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  }
}

template <int HPW>
constexpr size_t bulk_attn_smem() {
  return 2 * kStages * (size_t)kStagePos * kConsumerWarps * HPW * kHeadDim * 2 + 2 * kStages * 8 + 64;
}

// out[b, h, :] = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s. One CTA of kCombineWarps
// warps per (b, h): warp w folds splits w, w + kCombineWarps, ... with its own running
// max, then the warps merge through shared memory.
constexpr int kCombineWarps = 8;

__global__ void __launch_bounds__(kCombineWarps * 32)
attn_combine_kernel(const float* __restrict__ part_ml, const float* __restrict__ part_acc, int S,
                    __nv_bfloat16* __restrict__ out) {
  griddep_launch();
  griddep_wait();
  __shared__ float s_m[kCombineWarps], s_l[kCombineWarps];
  __shared__ float4 s_a[kCombineWarps][32];
  const int bh = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* ml = part_ml + 2 * (size_t)bh * S;
  const float* pa = part_acc + (size_t)bh * S * kHeadDim + 4 * lane;
  float M = -INFINITY;
  for (int s = warp + kCombineWarps * lane; s < S; s += kCombineWarps * 32) M = fmaxf(M, ml[2 * s]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
  float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
  for (int s = warp; s < S; s += kCombineWarps) {
    const float ms = ml[2 * s];
    const float f = ms == -INFINITY ? 0.f : expf(ms - M);
    L += ml[2 * s + 1] * f;
    const float4 a = *reinterpret_cast<const float4*>(pa + (size_t)s * kHeadDim);
    A.x += a.x * f;
    A.y += a.y * f;
    A.z += a.z * f;
    A.w += a.w * f;
  }
  if (lane == 0) {
    s_m[warp] = M;
    s_l[warp] = L;
  }
  s_a[warp][lane] = A;
  __syncthreads();
  if (warp != 0) return;
  float G = -INFINITY;
#pragma unroll
  for (int w = 0; w < kCombineWarps; ++w) G = fmaxf(G, s_m[w]);
  float LT = 0.f;
  float4 AT = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < kCombineWarps; ++w) {
    const float f = s_m[w] == -INFINITY ? 0.f : expf(s_m[w] - G);
    LT += s_l[w] * f;
    const float4 a = s_a[w][lane];
    AT.x += a.x * f;
    AT.y += a.y * f;
    AT.z += a.z * f;
    AT.w += a.w * f;
  }
  const float inv = LT > 0.f ? 1.0f / LT : 0.f;
  __nv_bfloat162 o2[2] = {__floats2bfloat162_rn(AT.x * inv, AT.y * inv),
                          __floats2bfloat162_rn(AT.z * inv, AT.w * inv)};
  *reinterpret_cast<uint2*>(out + (size_t)bh * kHeadDim + 4 * lane) = *reinterpret_cast<uint2*>(o2);
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
                                       const int32_t* block_table, int B, int max_blocks, int num_blocks, int NH,
                                       int D, int block_size, float theta, void* q_out, void* k_cache,
                                       void* v_cache, int* status, cudaStream_t stream) {
  if (B <= 0) return DWDP_OK;
  if (D % 2 || D > 1024 || block_size <= 0) return DWDP_ERR_INVALID_ARGUMENT;
  return launch_chained(rope_append_kernel, dim3((unsigned)B, (unsigned)NH), dim3(D / 2), 0, stream, 1u,
                        (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)bias, pos, block_table, max_blocks,
                        num_blocks, NH, D,
                        block_size, theta, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache,
                        reinterpret_cast<DeviceStatus*>(status)) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

static size_t acc_offset_floats(int B, int NH, int splits) {
  return ((size_t)B * NH * splits * 2 + 63) / 64 * 64;
}

extern "C" size_t dwdp_paged_attention_workspace_bytes_impl(int B, int NH, int splits) {
  return (acc_offset_floats(B, NH, splits) + (size_t)B * NH * splits * kHeadDim) * sizeof(float) + 256;
}

template <int HPW>
static cudaError_t launch_bulk_attn(dim3 grid, cudaStream_t stream, const __nv_bfloat16* q,
                                    const __nv_bfloat16* k, const __nv_bfloat16* v, const int32_t* table,
                                    const int32_t* lens, int max_blocks, int num_blocks, int block_size, int chunk,
                                    float scale, float* part_ml, float* part_acc, DeviceStatus* st) {
  constexpr size_t smem = bulk_attn_smem<HPW>();
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(paged_attn_bulk_kernel<HPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  return launch_chained(paged_attn_bulk_kernel<HPW>, grid, dim3((kConsumerWarps + 1) * 32), smem, stream, 1u, q, k, v,
                        table, lens, max_blocks, num_blocks, block_size, chunk, scale, part_ml, part_acc, st);
}

// splits: context chunks per sequence (per (sequence, head) on the fallback path);
// chunk = ceil(max_len / splits) positions, rounded up to a whole stage.
extern "C" int dwdp_paged_attention_launch(const void* q, const void* k_cache, const void* v_cache,
                                           const int32_t* block_table, const int32_t* seq_lens, int B,
                                           int max_blocks, int num_blocks, int NH, int D, int block_size,
                                           int max_len, int splits,
                                           float scale, void* workspace, void* out, int* status,
                                           cudaStream_t stream) {
  if (B <= 0) return DWDP_OK;
  if (D != kHeadDim || splits <= 0 || max_len <= 0) return DWDP_ERR_UNSUPPORTED;
  float* part_ml = reinterpret_cast<float*>(workspace);
  float* part_acc = part_ml + acc_offset_floats(B, NH, splits);
  DeviceStatus* st = reinterpret_cast<DeviceStatus*>(status);
  const bool aligned = ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u) == 0;
  const bool bulk = aligned && block_size % kStagePos == 0 && (NH == 8 || NH == 16 || NH == 32);
  cudaError_t e;
  if (bulk) {
    int chunk = (max_len + splits - 1) / splits;
    chunk = (chunk + kStagePos - 1) / kStagePos * kStagePos;
    const dim3 grid((unsigned)splits, (unsigned)B);
    const auto* qq = (const __nv_bfloat16*)q;
    const auto* kk = (const __nv_bfloat16*)k_cache;
    const auto* vv = (const __nv_bfloat16*)v_cache;
    e = NH == 8    ? launch_bulk_attn<1>(grid, stream, qq, kk, vv, block_table, seq_lens, max_blocks, num_blocks,
                                         block_size, chunk, scale, part_ml, part_acc, st)
        : NH == 16 ? launch_bulk_attn<2>(grid, stream, qq, kk, vv, block_table, seq_lens, max_blocks, num_blocks,
                                         block_size, chunk, scale, part_ml, part_acc, st)
                   : launch_bulk_attn<4>(grid, stream, qq, kk, vv, block_table, seq_lens, max_blocks, num_blocks,
                                         block_size, chunk, scale, part_ml, part_acc, st);
  } else {
    const int chunk = (max_len + splits - 1) / splits;
    e = launch_chained(paged_decode_attn_kernel, dim3((unsigned)B, (unsigned)NH, (unsigned)splits),
                       dim3(kAttnWarps * 32), 0, stream, 1u, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k_cache,
                       (const __nv_bfloat16*)v_cache, block_table, seq_lens, max_blocks, num_blocks, NH, block_size,
                       chunk, scale, part_ml, part_acc, st);
  }
  if (e != cudaSuccess) return DWDP_ERR_CUDA;
  const int BH = B * NH;
  return launch_chained(attn_combine_kernel, dim3((unsigned)BH), dim3(kCombineWarps * 32), 0, stream, 1u,
                        (const float*)part_ml, (const float*)part_acc, splits, (__nv_bfloat16*)out) ==
                 cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

// Grouped expert GEMMs on tcgen05 (sm_100a): the executor hot path.
//
// Replaces the per-expert loop of DWDP/executor/pytorch.py:66-160 (gather,
// down(silu(gate(x)) * up(x)), times routing weight) and the Triton persistent
// kernels of DWDP/executor/kernels/persistent.py:241-401 / fp8.py:147-318.
//
// Orientation ("swap AB"): the weight rows of one 128-row block are the MMA M
// dimension (TMEM lanes), the tokens of one expert tile are the MMA N dimension
// (16..128 columns, chosen per expert so a 273-row expert runs as 3 x 96, not
// 3 x 128). A per-output-channel or per-block weight scale therefore becomes a
// per-thread constant, and a decode step with one token per expert still fills
// the 128-row MMA with weights.
//
// Two launches per layer:
//   MODE 0  gate/up: acc_g, acc_u [128 feat x N tok] in TMEM (two MMAs sharing
//           the activation tile), epilogue h = silu(g) * u -> bf16 h[row, feat]
//   MODE 1  down   : acc [128 out x N tok], epilogue y * row_scale -> bf16 out
//
// Warp roles (one CTA per SM, persistent over a device-built work list):
//   warp 0      producer: one cp.async.bulk for the pre-tiled weight block(s)
//               + one TMA tile load of the activations per 64-wide K step
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-5   epilogue (TMEM lane quadrant = warp % 4), double-buffered acc
//   warps 6-13  (FP8 weights only) converter: e4m3 x scale -> bf16 into the
//               128B-swizzled operand image, then fence.proxy.async
// FP8 weights are multiplied as bf16 (e4m3 is exact in bf16; the fp32 scale is
// folded in with one rounding), so activations stay bf16: quantising them to
// e4m3 costs ~4.5% relative error, over the 2e-2 parity bar.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"

namespace dwdp {

#ifdef DWDP_PROFILE_ROLES
// Diagnostic build only: per-CTA cycle accounting of each role, written once at exit.
__device__ unsigned long long g_role_cycles[160][64];
#define PROF_DECL unsigned long long prof_[8] = {0, 0, 0, 0, 0, 0, 0, 0}; long long pt_ = 0; (void)pt_;
#define PROF_T0 pt_ = clock64();
#define PROF_ADD(i) prof_[i] += (unsigned long long)(clock64() - pt_);
#define PROF_STORE(base) { for (int q_ = 0; q_ < 4; ++q_) g_role_cycles[blockIdx.x][32 * MODE + 2 * (base) + q_] = prof_[q_]; g_role_cycles[blockIdx.x][32 * MODE + 2 * (base) + 4] = prof_[7]; }
#define TW(i, call) ([&]() { const long long t_ = clock64(); const bool r_ = (call); prof_[i] += (unsigned long long)(clock64() - t_); return r_; }())
#define PROF_START const long long pstart_ = clock64();
#define PROF_END(i) prof_[i] = (unsigned long long)(clock64() - pstart_);
#else
#define TW(i, call) (call)
#define PROF_START
#define PROF_END(i)
#define PROF_DECL
#define PROF_T0
#define PROF_ADD(i)
#define PROF_STORE(base) {}
#endif

constexpr int BM = 128;                    // weight rows per tile (MMA M)
constexpr int BK = 64;                     // K elements per pipeline stage (128 bytes of bf16)
constexpr int BN_MAX = 128;                // max tokens per tile (MMA N)
constexpr int kBTileBytes = BN_MAX * 128;  // activation tile: BN_MAX rows x 128 B
constexpr int kConvTileBytes = BM * 128;   // bf16 weight tile 128 x 64
constexpr int kFp8TileBytes = BM * BK;     // fp8 weight tile 128 x 64

struct WorkItem {
  int group;     // 0 routed, 1 shared
  int expert;    // expert index inside the group
  int rb;        // 128-row weight block
  int row0;      // first activation row of the tile
  int nrows;     // rows in this tile (<= BN_MAX)
  int kb_begin;  // first / one-past-last 64-wide K step of this item (split K)
  int kb_end;
  int part;      // K-split index: output goes to out + part * part_stride
  int nmat;      // weight matrices of the item: gate+up (2), or 1-2 consecutive down row blocks
  const uint8_t* wtiles;  // first weight tile of this item's 128-row block (set by the planner)
  const float* scales;    // the expert's scales (fp8) or nullptr
};

struct GroupParams {
  CUtensorMap tmap_b;      // activations [rows, K] bf16, box {64, BN_MAX}, 128B swizzle
  const void* const* w;    // [E] packed weight tiles
  const float* const* s;   // [E] scales (fp8) or nullptr
  void* out;               // bf16 [rows, R]
  const float* row_scale;  // MODE 1: per-row multiplier (routing weight / shared gate) or null
  const float* x_scale;    // e4m3 activation planes only: per-row activation scale
  int K;                   // reduction size
  int R;                   // output rows of the projection (= out leading dim)
  int scale_mode;
  int enabled;
  int box_rows;            // activation rows per TMA box (multiple of 16, <= BN_MAX)
  long long part_stride;   // elements between K-split partial outputs
  long long mstride;       // e4m3 path: bytes between an item's weight matrices
  long long kstride;       // e4m3 path: bytes between an item's 128-input stages
};

struct GemmParams {
  GroupParams g[2];
  const WorkItem* items;
  const int* n_items;
  int cap;  // work-item capacity (grid <= cap, so items[blockIdx.x] is always addressable)
  DeviceStatus* st;
};

template <int MODE, bool WFP8>
struct Cfg {
  static constexpr int NMAT = MODE == 0 ? 2 : 1;
  static constexpr int S = MODE == 0 ? 4 : 6;  // load stages
  static constexpr int CONV_GROUPS = 2;        // independent converter warp groups
  static constexpr int SC = WFP8 ? CONV_GROUPS : 0;  // converted-weight slots (one per group)
  static constexpr int W_STAGE_BYTES = NMAT * (WFP8 ? kFp8TileBytes : kConvTileBytes);
  static constexpr int CONV_STAGE_BYTES = NMAT * kConvTileBytes;
  static constexpr int NUM_WARPS = WFP8 ? 14 : 6;
  static constexpr int THREADS = NUM_WARPS * 32;
  static constexpr int CONV_THREADS = 256;
  static constexpr int TMEM_COLS = NMAT * BN_MAX * 2 <= 256 ? 256 : 512;
  static constexpr int ACC_STRIDE = NMAT * BN_MAX;  // TMEM columns per accumulator buffer
  static constexpr int SMEM_B = S * kBTileBytes;
  static constexpr int SMEM_W = S * W_STAGE_BYTES;
  static constexpr int SMEM_C = SC * CONV_STAGE_BYTES;
  static constexpr int SMEM_BYTES = SMEM_B + SMEM_W + SMEM_C + 1024 /*align*/ + 256 /*barriers*/;
};

// 16 e4m3 values of row r, elements [sub*16, sub*16+16) -> 32 bytes of bf16
// written to their 128B-swizzled positions.
// Four e4m3 bytes -> four bf16 (two words); exact unless `scaled` folds a block
// scale in (one rounding).
__device__ __forceinline__ void e4m3x4_to_bf16x4(uint32_t w, float s, bool scaled, uint32_t& o0, uint32_t& o1) {
  uint32_t out[2];
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((w >> (16 * hlf)) & 0xFFFFu);
    const __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
    const __nv_bfloat162 bv = scaled ? __floats2bfloat162_rn(f.x * s, f.y * s) : __floats2bfloat162_rn(f.x, f.y);
    out[hlf] = *reinterpret_cast<const uint32_t*>(&bv);
  }
  o0 = out[0];
  o1 = out[1];
}

// One 16-byte chunk (16 e4m3 of row r, elements [sub*16, sub*16+16)) -> 32 bytes
// of bf16 at their 128B-swizzled positions in the converted tile.
__device__ __forceinline__ void convert_chunk(const uint4 raw, uint8_t* conv_tile, int r, int sub, float s,
                                              bool scaled) {
  uint32_t o[8];
  e4m3x4_to_bf16x4(raw.x, s, scaled, o[0], o[1]);
  e4m3x4_to_bf16x4(raw.y, s, scaled, o[2], o[3]);
  e4m3x4_to_bf16x4(raw.z, s, scaled, o[4], o[5]);
  e4m3x4_to_bf16x4(raw.w, s, scaled, o[6], o[7]);
  const int c0 = sub * 2;  // 16-byte chunk index of the first 8 elements
  uint8_t* row = conv_tile + r * 128;
  *reinterpret_cast<uint4*>(row + ((c0 ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(row + (((c0 + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
}

template <int MODE, bool WFP8>
__global__ void __launch_bounds__(Cfg<MODE, WFP8>::THREADS, 1)
moe_gemm_kernel(const __grid_constant__ GemmParams p) {
  using C = Cfg<MODE, WFP8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sW = sB + C::SMEM_B;
  uint8_t* sC = sW + C::SMEM_W;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sC + C::SMEM_C);
  uint64_t* ld_full = bars;
  uint64_t* ld_empty = ld_full + C::S;
  uint64_t* cv_full = ld_empty + C::S;
  uint64_t* cv_empty = cv_full + 2;
  uint64_t* acc_full = cv_empty + 2;
  uint64_t* acc_empty = acc_full + 2;
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const int warp = warp_id();
  const int lane = lane_id();
  DeviceStatus* st = p.st;
  griddep_launch();

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < C::S; ++i) {
      mbar_init(&ld_full[i], 1);
      mbar_init(&ld_empty[i], WFP8 ? 2 : 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&cv_full[i], 1);
      mbar_init(&cv_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    if (p.g[0].enabled) prefetch_tmap(&p.g[0].tmap_b);
    if (p.g[1].enabled) prefetch_tmap(&p.g[1].tmap_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem_base;
  griddep_wait();  // the work list and operands come from the previous launches
  const int n_items = *p.n_items;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      PROF_DECL PROF_START
      uint32_t it = 0;
      WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
      for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
        const WorkItem wi = wn;
        if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
        const GroupParams& g = p.g[wi.group];
        const uint8_t* wbase = wi.wtiles;
        const uint32_t b_bytes = (uint32_t)g.box_rows * 128u;
        for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it) {
          const int s = it % C::S;
          if (!TW(0, mbar_wait(&ld_empty[s], ((it / C::S) & 1) ^ 1, &s_abort, st, 1 + 8 * MODE))) break;
          mbar_arrive_expect_tx(&ld_full[s], C::W_STAGE_BYTES + b_bytes);
          const size_t woff = (size_t)kb * C::W_STAGE_BYTES;
          bulk_g2s(sW + s * C::W_STAGE_BYTES, wbase + woff, C::W_STAGE_BYTES, &ld_full[s]);
          tma_load_2d(sB + s * kBTileBytes, &g.tmap_b, kb * BK, wi.row0, &ld_full[s]);
        }
      }
      PROF_END(7) PROF_STORE(0)
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      PROF_DECL PROF_START
      uint32_t it = 0, cit = 0;
      int li = 0;
      WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
      for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x, ++li) {
        const WorkItem wi = wn;
        if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
        const int a = li & 1;
        if (!TW(0, mbar_wait(&acc_empty[a], ((li >> 1) & 1) ^ 1, &s_abort, st, 2 + 8 * MODE))) break;
        tc_fence_after();
        const int n_mma = max(16, (wi.nrows + 15) & ~15);
        const uint32_t idesc = idesc_bf16(BM, n_mma);
        const uint32_t d_base = tmem_base + a * C::ACC_STRIDE;
        bool ok = true;
        for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it) {
          const int s = it % C::S;
          if (!TW(1, mbar_wait(&ld_full[s], (it / C::S) & 1, &s_abort, st, 3 + 8 * MODE))) { ok = false; break; }
          const uint8_t* wtile;
          int c = 0;
          if constexpr (WFP8) {
            c = cit % C::SC;
            if (!TW(2, mbar_wait(&cv_full[c], (cit / C::SC) & 1, &s_abort, st, 4 + 8 * MODE))) { ok = false; break; }
            wtile = sC + c * C::CONV_STAGE_BYTES;
          } else {
            wtile = sW + s * C::W_STAGE_BYTES;
          }
          tc_fence_after();
          // Descriptors are built once per stage; a K step of 16 bf16 (32 bytes) is +2 in
          // the encoded start address, the second weight matrix is +kConvTileBytes/16.
          const uint64_t b_desc0 = smem_desc_sw128(smem_u32(sB + s * kBTileBytes));
          const uint64_t a_desc0 = smem_desc_sw128(smem_u32(wtile));
          const uint32_t acc_first = kb > wi.kb_begin ? 1u : 0u;
          PROF_T0
#pragma unroll
          for (int m = 0; m < C::NMAT; ++m) {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              mma_bf16_ss(d_base + m * BN_MAX, a_desc0 + (uint64_t)(m * (kConvTileBytes >> 4) + 2 * kk),
                          b_desc0 + (uint64_t)(2 * kk), idesc, kk > 0 ? 1u : acc_first);
            }
          }
          PROF_ADD(3)
          mma_commit(&ld_empty[s]);
          if constexpr (WFP8) {
            mma_commit(&cv_empty[c]);
            ++cit;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[a]);
      }
      PROF_END(7) PROF_STORE(4)
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    PROF_DECL PROF_START
    const int quad = warp & 3;
    const int lrow = quad * 32 + lane;  // weight row inside the 128-row block
    int li = 0;
    WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
    for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x, ++li) {
      const WorkItem wi = wn;
      if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
      const GroupParams& g = p.g[wi.group];
      const int a = li & 1;
      const int feat = wi.rb * BM + lrow;
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)wi.part * g.part_stride;
      // per-output-channel weight scales are exact per-thread constants here (loaded while the MMAs run)
      float s0 = 1.0f, s1 = 1.0f;
      if (WFP8 && g.scale_mode == DWDP_SCALE_CHANNEL) {
        s0 = wi.scales[feat];
        if (MODE == 0) s1 = wi.scales[g.R + feat];
      }
      if (!TW(0, mbar_wait(&acc_full[a], (li >> 1) & 1, &s_abort, st, 5 + 8 * MODE))) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + a * C::ACC_STRIDE + ((uint32_t)(quad * 32) << 16);
      for (int c0 = 0; c0 < wi.nrows; c0 += 16) {
        if constexpr (MODE == 0) {
          float gv[16], uv[16];
          tmem_ld16(t_acc + c0, gv);
          tmem_ld16(t_acc + BN_MAX + c0, uv);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            if (col < wi.nrows) {
              const float h = silu(gv[j] * s0) * (uv[j] * s1);
              out[(size_t)(wi.row0 + col) * g.R + feat] = __float2bfloat16_rn(h);
            }
          }
        } else {
          float yv[16];
          tmem_ld16(t_acc + c0, yv);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            if (col < wi.nrows) {
              const int row = wi.row0 + col;
              const float sc = g.row_scale != nullptr ? g.row_scale[row] : 1.0f;
              out[(size_t)row * g.R + feat] = __float2bfloat16_rn(yv[j] * s0 * sc);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
    PROF_END(7) if (lane == 0 && quad == 0) PROF_STORE(8)
  } else if constexpr (WFP8) {
    // ------------------------------------------------------------ converter (fp8 -> bf16)
    // CHANNEL scales are applied in the epilogue, so the conversion is exact
    // (e4m3 values are representable in bf16); BLOCK128 scales vary with K and
    // are folded in here with one rounding.
    // The converter warps form C::CONV_GROUPS independent groups; group g converts
    // the stages with index % CONV_GROUPS == g into conversion slot g, so several
    // stages convert at once (conversion is latency-, not throughput-bound).
    PROF_DECL PROF_START
    const int ct = threadIdx.x - 6 * 32;  // 0..255
    constexpr int kGroupThreads = C::CONV_THREADS / C::CONV_GROUPS;
    const int grp = ct / kGroupThreads, gt = ct % kGroupThreads;
    uint32_t it = 0, cit = 0;
    WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
    for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
      const WorkItem wi = wn;
      if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
      const GroupParams& g = p.g[wi.group];
      const bool block_scaled = g.scale_mode == DWDP_SCALE_BLOCK128;
      const float* sc = wi.scales;
      bool ok = true;
      for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it, ++cit) {
        if ((int)(cit % C::CONV_GROUPS) != grp) continue;
        const int s = it % C::S;
        const int c = cit % C::SC;
        float sblk[C::NMAT];
#pragma unroll
        for (int m = 0; m < C::NMAT; ++m)
          sblk[m] = block_scaled ? sc[((size_t)m * (g.R / 128) + wi.rb) * (g.K / 128) + (kb >> 1)] : 1.0f;
        if (!TW(0, mbar_wait(&ld_full[s], (it / C::S) & 1, &s_abort, st, 6 + 8 * MODE))) { ok = false; break; }
        if (!TW(1, mbar_wait(&cv_empty[c], ((cit / C::SC) & 1) ^ 1, &s_abort, st, 7 + 8 * MODE))) { ok = false; break; }
        const uint8_t* raw = sW + s * C::W_STAGE_BYTES;
        uint8_t* conv = sC + c * C::CONV_STAGE_BYTES;
        constexpr int kChunks = C::NMAT * kFp8TileBytes / 16;  // 16-byte chunks per stage
        constexpr int kPer = kChunks / kGroupThreads;          // chunks per converter thread
        uint4 rawv[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {  // issue every shared load first
          const int q = gt + j * kGroupThreads;
          const int m = q / (kFp8TileBytes / 16), rem = q % (kFp8TileBytes / 16);
          rawv[j] = *reinterpret_cast<const uint4*>(raw + m * kFp8TileBytes + (rem >> 2) * BK + (rem & 3) * 16);
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int q = gt + j * kGroupThreads;
          const int m = q / (kFp8TileBytes / 16), rem = q % (kFp8TileBytes / 16);
          convert_chunk(rawv[j], conv + m * kConvTileBytes, rem >> 2, rem & 3, sblk[m], block_scaled);
        }
        fence_proxy_async_smem();
        named_bar_sync(1 + grp, kGroupThreads);
        if (gt == 0) {
          mbar_arrive(&cv_full[c]);
          mbar_arrive(&ld_empty[s]);
        }
      }
      if (!ok) break;
    }
    PROF_END(7) if (ct == 0) PROF_STORE(12)
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// hi/lo activation planes: lo = (v / s - hi) * kLoPlaneGain (see quant_rows)
constexpr float kLoPlaneGain = 16.0f;

// ---------------------------------------------------------------------------
// e4m3 tensor-core path (per-output-channel fp8 weights).
//
// The weights are multiplied as e4m3 by tcgen05 kind::f8f6f4 straight from the
// pre-swizzled 128 x 128 tiles the bulk copy lands in shared memory: no
// conversion warps, and one MMA covers 32 inputs (twice a bf16 MMA). The
// activations come as hi/lo e4m3 planes (interleaved rows, see quant_rows), so
// the MMA N dimension holds 2 columns per token and the epilogue forms
//   y = s_w[row] * s_x[token] * (acc[2t] + acc[2t + 1] / 16)
// which keeps bf16-level activation precision. Token tiles are at most 64
// (N <= 128), so two accumulator buffers of gate+up fit the 512 TMEM columns.
// Warp roles: 0 producer, 1 TMEM allocator + MMA issuer, 2-5 epilogue.
// ---------------------------------------------------------------------------
constexpr int BK8 = 128;                    // e4m3 inputs per pipeline stage
constexpr int BN8 = 64;                     // max tokens per tile
constexpr int kW8TileBytes = BM * BK8;      // 128 x 128 weight tile

// NM = weight matrices per stage: 2 for gate+up or paired down row blocks, 1 for single down blocks.
// BNT = tokens per tile (64 at decode sizes, 128 at prefill sizes: twice the MMA work per weight
// byte). An accumulator buffer holds NM x 2 x BNT columns; two buffers when they fit TMEM's 512.
template <int MODE, int NM, int BNT>
struct Cfg8 {
  static constexpr int NMAT = NM;
  static constexpr int B_TILE = 2 * BNT * BK8;                 // hi/lo activation tile
  static constexpr int W_STAGE_BYTES = NMAT * kW8TileBytes;
  static constexpr int OUT_COLS = MODE == 0 ? BM : NMAT * BM;  // output features per item
  static constexpr int STAGING = BNT * OUT_COLS * 2;            // bf16 [tokens][features] epilogue tile
  static constexpr int S = (224 * 1024 - STAGING) / (W_STAGE_BYTES + B_TILE);
  static constexpr int EPI_WARPS = 8;  // two warps per TMEM lane quadrant, alternate column chunks
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int THREADS = (2 + EPI_WARPS) * 32;
  static constexpr int ACC_STRIDE = NMAT * 2 * BNT;            // TMEM columns per accumulator buffer
  static constexpr int NBUF = 2 * ACC_STRIDE <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = NBUF * ACC_STRIDE <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = S * (W_STAGE_BYTES + B_TILE) + STAGING + 1024 + 256;
};

template <int MODE, int NM, int BNT>
__global__ void __launch_bounds__(Cfg8<MODE, NM, BNT>::THREADS, 1)
moe_gemm_f8_kernel(const __grid_constant__ GemmParams p) {
  using C = Cfg8<MODE, NM, BNT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sW = sB + C::S * C::B_TILE;
  __nv_bfloat16* sOut = reinterpret_cast<__nv_bfloat16*>(sW + C::S * C::W_STAGE_BYTES);  // [BNT][OUT_COLS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sOut) + C::STAGING);
  uint64_t* ld_full = bars;
  uint64_t* ld_empty = ld_full + C::S;
  uint64_t* acc_full = ld_empty + C::S;
  uint64_t* acc_empty = acc_full + 2;
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const int warp = warp_id();
  const int lane = lane_id();
  DeviceStatus* st = p.st;
  griddep_launch();

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < C::S; ++i) {
      mbar_init(&ld_full[i], 1);
      mbar_init(&ld_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], C::EPI_THREADS);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    if (p.g[0].enabled) prefetch_tmap(&p.g[0].tmap_b);
    if (p.g[1].enabled) prefetch_tmap(&p.g[1].tmap_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem_base;
  griddep_wait();  // the work list and operands come from the previous launches
  const int n_items = *p.n_items;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      PROF_DECL PROF_START
      uint32_t it = 0;
      WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
      for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
        const WorkItem wi = wn;
        if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
        const GroupParams& g = p.g[wi.group];
        const uint8_t* wbase = wi.wtiles;
        const uint32_t b_bytes = (uint32_t)g.box_rows * 2u * BK8;
        for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it) {
          const int s = it % C::S;
          if (!TW(0, mbar_wait(&ld_empty[s], ((it / C::S) & 1) ^ 1, &s_abort, st, 21 + 8 * MODE))) break;
          const int nm = min(wi.nmat, C::NMAT);
          mbar_arrive_expect_tx(&ld_full[s], (uint32_t)(nm * kW8TileBytes) + b_bytes);
          for (int m = 0; m < nm; ++m)
            bulk_g2s(sW + s * C::W_STAGE_BYTES + m * kW8TileBytes,
                     wbase + (size_t)m * g.mstride + (size_t)kb * g.kstride, kW8TileBytes, &ld_full[s]);
          tma_load_2d(sB + s * C::B_TILE, &g.tmap_b, kb * BK8, 2 * wi.row0, &ld_full[s]);
        }
      }
      PROF_END(7) PROF_STORE(0)
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      PROF_DECL PROF_START
      uint32_t it = 0;
      int li = 0;
      WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
      for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x, ++li) {
        const WorkItem wi = wn;
        if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
        const int a = li % C::NBUF;
        if (!TW(0, mbar_wait(&acc_empty[a], ((li / C::NBUF) & 1) ^ 1, &s_abort, st, 22 + 8 * MODE))) break;
        tc_fence_after();
        const int n_tok = max(16, (wi.nrows + 15) & ~15);
        const uint32_t idesc = idesc_e4m3(BM, 2 * n_tok);
        const uint32_t d_base = tmem_base + a * C::ACC_STRIDE;
        bool ok = true;
        for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it) {
          const int s = it % C::S;
          if (!TW(1, mbar_wait(&ld_full[s], (it / C::S) & 1, &s_abort, st, 23 + 8 * MODE))) { ok = false; break; }
          tc_fence_after();
          // a K step of 32 e4m3 (32 bytes) is +2 in the encoded start address
          const uint64_t b_desc0 = smem_desc_sw128(smem_u32(sB + s * C::B_TILE));
          const uint64_t a_desc0 = smem_desc_sw128(smem_u32(sW + s * C::W_STAGE_BYTES));
          const uint32_t acc_first = kb > wi.kb_begin ? 1u : 0u;
          PROF_T0
          for (int m = 0; m < min(wi.nmat, C::NMAT); ++m) {
#pragma unroll
            for (int kk = 0; kk < BK8 / 32; ++kk) {
              mma_e4m3_ss(d_base + m * 2 * BNT, a_desc0 + (uint64_t)(m * (kW8TileBytes >> 4) + 2 * kk),
                          b_desc0 + (uint64_t)(2 * kk), idesc, kk > 0 ? 1u : acc_first);
            }
          }
          PROF_ADD(3)
          mma_commit(&ld_empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[a]);
      }
      PROF_END(7) PROF_STORE(4)
    }
  } else {
    // ------------------------------------------------------------ epilogue
    PROF_DECL PROF_START
    const int quad = warp & 3;
    const int lrow = quad * 32 + lane;
    const int eg = (warp - 2) >> 2;        // epilogue group (0, 1)
    const int ep = (warp - 2) * 32 + lane;  // 0 .. EPI_THREADS - 1
    int li = 0;
    WorkItem wn = p.items[blockIdx.x];  // fetched with n_items; the next one is prefetched
    for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x, ++li) {
      const WorkItem wi = wn;
      if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
      const GroupParams& g = p.g[wi.group];
      const int a = li % C::NBUF;
      const int feat = wi.rb * BM + lrow;
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)wi.part * g.part_stride;
      // gate/up: s0, s1 scale the two matrices of one feature; down: two consecutive features
      const float s0 = wi.scales[feat];  // loaded while the MMAs run
      const int nmat = min(wi.nmat, C::NMAT);
      const float s1 = MODE == 0 ? wi.scales[g.R + feat] : (nmat > 1 ? wi.scales[feat + BM] : 1.0f);
      const float* xs = g.x_scale + wi.row0;
      if (!TW(0, mbar_wait(&acc_full[a], (li / C::NBUF) & 1, &s_abort, st, 24 + 8 * MODE))) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + a * C::ACC_STRIDE + ((uint32_t)(quad * 32) << 16);
      // Small tiles (decode) store straight from registers; larger ones go through the bf16
      // staging tile so that the accumulator is released as soon as TMEM is drained and the
      // rows leave as 16-byte stores. The two warps of a lane quadrant take alternate
      // 32-column (16-token) chunks.
      const bool direct = wi.nrows <= 16;
      for (int c0 = eg * 32; c0 < 2 * wi.nrows; c0 += 64) {
        const int t0 = c0 >> 1;
        if constexpr (MODE == 0) {
          float gv[32], uv[32];
          tmem_ld32(t_acc + c0, gv);
          tmem_ld32(t_acc + 2 * BNT + c0, uv);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = t0 + j;
            if (t < wi.nrows) {
              const float sx = xs[t];
              const float gg = (gv[2 * j] + gv[2 * j + 1] * (1.0f / kLoPlaneGain)) * (s0 * sx);
              const float uu = (uv[2 * j] + uv[2 * j + 1] * (1.0f / kLoPlaneGain)) * (s1 * sx);
              const __nv_bfloat16 h = __float2bfloat16_rn(silu_fast(gg) * uu);
              if (direct) out[(size_t)(wi.row0 + t) * g.R + feat] = h;
              else sOut[t * C::OUT_COLS + lrow] = h;
            }
          }
        } else {
          float yv[C::NMAT][32];
#pragma unroll
          for (int m = 0; m < C::NMAT; ++m)
            if (m < nmat) tmem_ld32(t_acc + m * 2 * BNT + c0, yv[m]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = t0 + j;
            if (t < wi.nrows) {
              const float f = xs[t] * (g.row_scale != nullptr ? g.row_scale[wi.row0 + t] : 1.0f);
#pragma unroll
              for (int m = 0; m < C::NMAT; ++m) {
                if (m < nmat) {
                  const float y = (yv[m][2 * j] + yv[m][2 * j + 1] * (1.0f / kLoPlaneGain)) * ((m == 0 ? s0 : s1) * f);
                  const __nv_bfloat16 yb = __float2bfloat16_rn(y);
                  if (direct) out[(size_t)(wi.row0 + t) * g.R + feat + m * BM] = yb;
                  else sOut[t * C::OUT_COLS + m * BM + lrow] = yb;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
      if (!direct) {
        named_bar_sync(3, C::EPI_THREADS);
        const int cols = MODE == 0 ? BM : nmat * BM;  // features of this item
        const int cpr = cols / 8;                      // 16-byte chunks per token row
        for (int q = ep; q < wi.nrows * cpr; q += C::EPI_THREADS) {
          const int t = q / cpr, ch = q - t * cpr;
          const uint4 v = *reinterpret_cast<const uint4*>(sOut + t * C::OUT_COLS + ch * 8);
          *reinterpret_cast<uint4*>(out + (size_t)(wi.row0 + t) * g.R + wi.rb * BM + ch * 8) = v;
        }
        named_bar_sync(3, C::EPI_THREADS);  // the staging tile is rewritten by the next item
      }
    }
    PROF_END(7) if (lane == 0 && quad == 0) PROF_STORE(8)
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Device tile planner (the scheduler's job, DWDP/scheduler/ops/round_robin.py:
// active experts in ascending id), run on device so no counts reach the host.
// Shared-expert tiles go first (longest-running work first); routed tiles are
// ordered (expert, weight block, token tile) so CTAs running at the same time
// stream the same weight blocks through L2.
// ---------------------------------------------------------------------------
struct PlanParams {
  const int64_t* counts;
  const int64_t* offsets;
  int E, T, has_shared;
  int rb_gu_r, rb_dn_r, rb_gu_s, rb_dn_s;  // 128-row weight blocks per projection
  int kb_gu, kb_dn_r, kb_dn_s;              // 64-wide K steps per projection
  int sdn_parts;                            // K splits of the shared down projection
  int bn_max;                               // token-tile cap (rows per work item)
  const void* const* w_gu[2];               // [group] per-expert weight slabs (routed, shared)
  const void* const* w_dn[2];
  const float* const* s_gu[2];              // [group] per-expert scales (or nullptr)
  const float* const* s_dn[2];
  long long rbb_gu[2], rbb_dn[2];           // bytes of one 128-row weight block
  int dn_pair;                              // down items cover two consecutive 128-row blocks
  int blocks_dn;                            // 128-row blocks of the down projection (H / 128)
  WorkItem* items_gu;
  WorkItem* items_dn;
  int* n_items;
  int cap_gu, cap_dn;
  DeviceStatus* st;
};

constexpr int kPlanThreads = 256;
constexpr int kPlanBlocks = 64;

// Multi-CTA planner: every CTA rebuilds the (small) per-expert tile prefix in
// shared memory, then writes its slice of the flat work-item index space of both
// phases. Items are (shared tiles) followed by (expert ascending, weight block,
// token tile); an item's expert is found by binary search over the prefix.
__device__ __forceinline__ void plan_body(const PlanParams& pp) {
  __shared__ int s_pre[1025];   // exclusive prefix of token tiles per expert
  __shared__ int s_bn[1024];    // rows per tile of each expert
  __shared__ int s_nt[1024];    // token tiles of each expert
  __shared__ int s_part[kPlanThreads];
  const int tid = threadIdx.x;
  const int T = pp.T, E = pp.E;
  // per-expert tiles, scanned in chunks of kPlanThreads * 4
  int carry = 0;
  for (int e0 = 0; e0 < E; e0 += kPlanThreads * 4) {
    int loc[4], sum = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = e0 + tid * 4 + q;
      int nt = 0, bn = 0;
      if (e < E) {
        const int cnt = pp.counts != nullptr ? (int)pp.counts[e] : 0;
        if (cnt > 0) {
          nt = (cnt + pp.bn_max - 1) / pp.bn_max;
          bn = (((cnt + nt - 1) / nt) + 15) & ~15;
        }
        s_nt[e] = nt;
        s_bn[e] = bn;
      }
      loc[q] = nt;
      sum += nt;
    }
    s_part[tid] = sum;
    __syncthreads();
    for (int o = 1; o < kPlanThreads; o <<= 1) {
      const int add = tid >= o ? s_part[tid - o] : 0;
      __syncthreads();
      s_part[tid] += add;
      __syncthreads();
    }
    int run = carry + s_part[tid] - sum;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = e0 + tid * 4 + q;
      if (e < E) s_pre[e] = run;
      run += loc[q];
    }
    const int total = s_part[kPlanThreads - 1];
    __syncthreads();
    carry += total;
  }
  if (tid == 0) s_pre[E] = carry;
  __syncthreads();
  const int routed_tiles = carry;

  int n_sh_tiles = 0, bn_s = 0;
  if (pp.has_shared && T > 0) {
    n_sh_tiles = (T + pp.bn_max - 1) / pp.bn_max;
    bn_s = (((T + n_sh_tiles - 1) / n_sh_tiles) + 15) & ~15;
  }
  const int base_gu = n_sh_tiles * pp.rb_gu_s;
  const int base_dn = n_sh_tiles * pp.rb_dn_s * pp.sdn_parts;
  const int ngu = base_gu + routed_tiles * pp.rb_gu_r;
  const int ndn = base_dn + routed_tiles * pp.rb_dn_r;
  if (ngu > pp.cap_gu || ndn > pp.cap_dn) {
    if (blockIdx.x == 0 && tid == 0) {
      record_error(pp.st, DWDP_ERR_CAPACITY, 200, ngu);
      pp.n_items[0] = 0;
      pp.n_items[1] = 0;
    }
    return;
  }
  if (blockIdx.x == 0 && tid == 0) {
    pp.n_items[0] = ngu;
    pp.n_items[1] = ndn;
  }
  const int kb_part = pp.sdn_parts > 0 ? pp.kb_dn_s / pp.sdn_parts : 0;
  const int stride = kPlanBlocks * kPlanThreads;
  for (int phase = 0; phase < 2; ++phase) {
    const int n = phase == 0 ? ngu : ndn;
    const int base = phase == 0 ? base_gu : base_dn;
    const int rb_r = phase == 0 ? pp.rb_gu_r : pp.rb_dn_r;
    const int kb_r = phase == 0 ? pp.kb_gu : pp.kb_dn_r;
    WorkItem* out = phase == 0 ? pp.items_gu : pp.items_dn;
    for (int i = blockIdx.x * blockDim.x + tid; i < n; i += stride) {
      WorkItem w;
      if (i < base) {  // shared expert: (part, rb, token tile)
        const int per_part = n_sh_tiles * (phase == 0 ? pp.rb_gu_s : pp.rb_dn_s);
        const int part = phase == 0 ? 0 : i / per_part;
        const int rem = phase == 0 ? i : i % per_part;
        const int rbi = rem / n_sh_tiles, j = rem % n_sh_tiles;
        const int rb = (phase == 1 && pp.dn_pair) ? 2 * rbi : rbi;
        const int row0 = j * bn_s;
        const int kb0 = phase == 0 ? 0 : part * kb_part;
        const int kb1 = phase == 0 ? pp.kb_gu : (part + 1) * kb_part;
        w = WorkItem{1, 0, rb, row0, min(bn_s, T - row0), kb0, kb1, part, 2, nullptr, nullptr};
      } else {         // routed: expert e with s_pre[e]*rb_r <= i - base < s_pre[e+1]*rb_r
        const int r = i - base;
        int lo = 0, hi = E - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_pre[mid] * rb_r <= r) lo = mid; else hi = mid - 1;
        }
        const int e = lo;
        const int nt = s_nt[e], bn = s_bn[e];
        const int local = r - s_pre[e] * rb_r;
        const int rbi = local / nt, j = local % nt;
        const int rb = (phase == 1 && pp.dn_pair) ? 2 * rbi : rbi;
        const int cnt = (int)pp.counts[e];
        const int row0 = (int)pp.offsets[e] + j * bn;
        w = WorkItem{0, e, rb, row0, min(bn, cnt - j * bn), 0, kb_r, 0, 2, nullptr, nullptr};
      }
      if (phase == 1) w.nmat = pp.dn_pair ? min(2, pp.blocks_dn - w.rb) : 1;
      const void* const* wp = phase == 0 ? pp.w_gu[w.group] : pp.w_dn[w.group];
      const float* const* sp = phase == 0 ? pp.s_gu[w.group] : pp.s_dn[w.group];
      const long long rbb = phase == 0 ? pp.rbb_gu[w.group] : pp.rbb_dn[w.group];
      w.wtiles = reinterpret_cast<const uint8_t*>(wp[w.expert]) + (size_t)w.rb * rbb;
      w.scales = sp != nullptr ? sp[w.expert] : nullptr;
      out[i] = w;
    }
  }
}

// ---------------------------------------------------------------------------
// Activation planes for the e4m3 tensor-core path. A bf16 row v[0..K) becomes
// two e4m3 rows with one fp32 scale s = amax / 448:
//   hi = e4m3(v / s),  lo = e4m3((v / s - hi) * 16),  v ~= s * (hi + lo / 16)
// (about 8 significant bits, like bf16). The planes are stored interleaved,
// row 2i = hi of row i, row 2i + 1 = lo of row i, so one TMA box brings both
// and the MMA's N columns alternate hi/lo per token.
// ---------------------------------------------------------------------------
struct QuantSeg {
  const __nv_bfloat16* src;  // [src_rows, K]
  uint8_t* dst;              // [2 * rows, K]
  float* scale;              // [rows]
  int rows, K;
  const int64_t* row_index;  // row r reads src row row_index[r] (null: row r)
  int64_t src_rows;
};
struct QuantParams {
  QuantSeg seg[2];
  DeviceStatus* st;
  int per_warp;  // 1: one warp per row (many rows); 0: one CTA per row (few, long rows)
};

// 8 bf16 (one 16-byte load) -> 8 hi bytes and 8 lo bytes
__device__ __forceinline__ void quant8(const uint4 v, float inv, uint2& hi8, uint2& lo8) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
  uint32_t h[2] = {0, 0}, l[2] = {0, 0};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(b[q]);
    const float2 xs = make_float2(f.x * inv, f.y * inv);
    const __nv_fp8x2_storage_t hq = __nv_cvt_float2_to_fp8x2(xs, __NV_SATFINITE, __NV_E4M3);
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(hq, __NV_E4M3);
    const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const float2 r = make_float2((xs.x - hf.x) * kLoPlaneGain, (xs.y - hf.y) * kLoPlaneGain);
    const __nv_fp8x2_storage_t lq = __nv_cvt_float2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
    h[q >> 1] |= (uint32_t)hq << (16 * (q & 1));
    l[q >> 1] |= (uint32_t)lq << (16 * (q & 1));
  }
  hi8 = make_uint2(h[0], h[1]);
  lo8 = make_uint2(l[0], l[1]);
}

__device__ __forceinline__ float amax8(const uint4 v, float m) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(b[q]);
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

// One CTA (kPlanThreads threads) quantises one row: every 16-byte load of the
// row is issued before the amax reduction (rows up to kQuantRegChunks * 2048
// elements stay in registers; longer rows re-read their tail), so a row costs
// about one memory latency.
constexpr int kQuantRegChunks = 4;

__device__ __forceinline__ void quant_row_block(const QuantSeg& g, int row, float* red, DeviceStatus* st) {
  const int tid = threadIdx.x;
  int64_t sr = row;
  if (g.row_index != nullptr) {
    sr = g.row_index[row];
    if (sr < 0 || sr >= g.src_rows) {  // bad index: record it, quantise a zero row
      if (tid == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 210, row);
      sr = -1;
    }
  }
  const __nv_bfloat16* src = sr >= 0 ? g.src + (size_t)sr * g.K : nullptr;
  const int K = src != nullptr ? g.K : 0;  // a zero row reads nothing
  constexpr int kStride = kPlanThreads * 8;
  uint4 v[kQuantRegChunks];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kQuantRegChunks; ++j) {
    const int c = j * kStride + tid * 8;
    v[j] = c < K ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < kQuantRegChunks; ++j) amax = amax8(v[j], amax);
  for (int c = kQuantRegChunks * kStride + tid * 8; c < K; c += kStride)
    amax = amax8(*reinterpret_cast<const uint4*>(src + c), amax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < kPlanThreads / 32; ++i) amax = fmaxf(amax, red[i]);
  __syncthreads();  // red is reused by the next row
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  uint8_t* hi = g.dst + (size_t)(2 * row) * g.K;
  uint8_t* lo = hi + g.K;
#pragma unroll
  for (int j = 0; j < kQuantRegChunks; ++j) {
    const int c = j * kStride + tid * 8;
    if (c < g.K) {
      uint2 h8, l8;
      quant8(v[j], inv, h8, l8);
      *reinterpret_cast<uint2*>(hi + c) = h8;
      *reinterpret_cast<uint2*>(lo + c) = l8;
    }
  }
  for (int c = kQuantRegChunks * kStride + tid * 8; c < g.K; c += kStride) {
    uint2 h8, l8;
    quant8(K > 0 ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0), inv, h8, l8);
    *reinterpret_cast<uint2*>(hi + c) = h8;
    *reinterpret_cast<uint2*>(lo + c) = l8;
  }
  if (tid == 0) g.scale[row] = amax > 0.f ? amax / 448.0f : 0.f;
}

// One warp quantises one row: the first 8 chunks of 16 bytes per lane (rows up
// to 2048 elements) stay in registers, longer rows re-read their tail.
__device__ __forceinline__ void quant_row_warp(const QuantSeg& g, int row, DeviceStatus* st) {
  const int lane = threadIdx.x & 31;
  int64_t sr = row;
  if (g.row_index != nullptr) {
    sr = g.row_index[row];
    if (sr < 0 || sr >= g.src_rows) {
      if (lane == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 211, row);
      sr = -1;
    }
  }
  const __nv_bfloat16* src = sr >= 0 ? g.src + (size_t)sr * g.K : nullptr;
  const int K = src != nullptr ? g.K : 0;
  constexpr int kC = 8;
  uint4 v[kC];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kC; ++j) {
    const int c = (j * 32 + lane) * 8;
    v[j] = c < K ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < kC; ++j) amax = amax8(v[j], amax);
  for (int c = (kC * 32 + lane) * 8; c < K; c += 256) amax = amax8(*reinterpret_cast<const uint4*>(src + c), amax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  uint8_t* hi = g.dst + (size_t)(2 * row) * g.K;
  uint8_t* lo = hi + g.K;
#pragma unroll
  for (int j = 0; j < kC; ++j) {
    const int c = (j * 32 + lane) * 8;
    if (c < g.K) {
      uint2 h8, l8;
      quant8(v[j], inv, h8, l8);
      *reinterpret_cast<uint2*>(hi + c) = h8;
      *reinterpret_cast<uint2*>(lo + c) = l8;
    }
  }
  for (int c = (kC * 32 + lane) * 8; c < g.K; c += 256) {
    uint2 h8, l8;
    quant8(K > 0 ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0), inv, h8, l8);
    *reinterpret_cast<uint2*>(hi + c) = h8;
    *reinterpret_cast<uint2*>(lo + c) = l8;
  }
  if (lane == 0) g.scale[row] = amax > 0.f ? amax / 448.0f : 0.f;
}

// As quant_row_warp for rows whose width is a multiple of 16: a lane takes 16 consecutive
// elements per step (two 16-byte loads, one 16-byte store per plane) instead of 8.
__device__ __forceinline__ void quant_row_warp16(const QuantSeg& g, int row, DeviceStatus* st) {
  const int lane = threadIdx.x & 31;
  int64_t sr = row;
  if (g.row_index != nullptr) {
    sr = g.row_index[row];
    if (sr < 0 || sr >= g.src_rows) {
      if (lane == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 212, row);
      sr = -1;
    }
  }
  const __nv_bfloat16* src = sr >= 0 ? g.src + (size_t)sr * g.K : nullptr;
  const int K = src != nullptr ? g.K : 0;
  constexpr int kP = 4;  // 16-element steps kept in registers (rows up to 2048)
  uint4 v[2 * kP];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kP; ++j) {
    const int c = (j * 32 + lane) * 16;
    v[2 * j] = c < K ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
    v[2 * j + 1] = c < K ? *reinterpret_cast<const uint4*>(src + c + 8) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < 2 * kP; ++j) amax = amax8(v[j], amax);
  for (int c = (kP * 32 + lane) * 16; c < K; c += 512) {
    amax = amax8(*reinterpret_cast<const uint4*>(src + c), amax);
    amax = amax8(*reinterpret_cast<const uint4*>(src + c + 8), amax);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  uint8_t* hi = g.dst + (size_t)(2 * row) * g.K;
  uint8_t* lo = hi + g.K;
  auto put = [&](const uint4 a, const uint4 b, int c) {
    uint2 ha, la, hb, lb;
    quant8(a, inv, ha, la);
    quant8(b, inv, hb, lb);
    *reinterpret_cast<uint4*>(hi + c) = make_uint4(ha.x, ha.y, hb.x, hb.y);
    *reinterpret_cast<uint4*>(lo + c) = make_uint4(la.x, la.y, lb.x, lb.y);
  };
#pragma unroll
  for (int j = 0; j < kP; ++j) {
    const int c = (j * 32 + lane) * 16;
    if (c < g.K) put(v[2 * j], v[2 * j + 1], c);
  }
  for (int c = (kP * 32 + lane) * 16; c < g.K; c += 512) {
    const uint4 a = K > 0 ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
    const uint4 b = K > 0 ? *reinterpret_cast<const uint4*>(src + c + 8) : make_uint4(0, 0, 0, 0);
    put(a, b, c);
  }
  if (lane == 0) g.scale[row] = amax > 0.f ? amax / 448.0f : 0.f;
}

// Rows of both segments, one per `first + i * stride` unit (a warp or a CTA).
__device__ __forceinline__ void quant_rows(const QuantParams& q, int block, int nblocks) {
  __shared__ float red[kPlanThreads / 32];
  const int total = q.seg[0].rows + q.seg[1].rows;
  if (q.per_warp) {
    constexpr int kW = kPlanThreads / 32;
    for (int r = block * kW + (int)(threadIdx.x >> 5); r < total; r += nblocks * kW) {
      const QuantSeg& sg = r < q.seg[0].rows ? q.seg[0] : q.seg[1];
      const int rr = r < q.seg[0].rows ? r : r - q.seg[0].rows;
      if (sg.K % 16 == 0) quant_row_warp16(sg, rr, q.st);
      else quant_row_warp(sg, rr, q.st);
    }
    return;
  }
  for (int r = block; r < total; r += nblocks) {
    if (r < q.seg[0].rows) quant_row_block(q.seg[0], r, red, q.st);
    else quant_row_block(q.seg[1], r - q.seg[0].rows, red, q.st);
  }
}

// One launch before the gate/up GEMM: blocks [0, kPlanBlocks) build the work
// lists, the rest quantise the activation rows (when the e4m3 path runs).
__global__ void __launch_bounds__(kPlanThreads) prep_kernel(const PlanParams pp, const QuantParams qp) {
  griddep_launch();
  griddep_wait();
  if (blockIdx.x < kPlanBlocks) {
    plan_body(pp);
    return;
  }
  quant_rows(qp, blockIdx.x - kPlanBlocks, gridDim.x - kPlanBlocks);
}

// Quantisation of the SwiGLU intermediate rows between the two GEMMs.
__global__ void __launch_bounds__(kPlanThreads) quant_kernel(const QuantParams qp) {
  griddep_launch();
  griddep_wait();
  quant_rows(qp, blockIdx.x, gridDim.x);
}

}  // namespace dwdp

using namespace dwdp;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box {64, BN_MAX}, 128B swizzle.
bool make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto enc = get_encode_fn();
  if (enc == nullptr || rows <= 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D map over the interleaved hi/lo e4m3 planes [2 * rows, cols], box {128, 2 * box_rows}.
bool make_tmap_planes(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto enc = get_encode_fn();
  if (enc == nullptr || rows <= 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)(2 * rows)};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)BK8, (cuuint32_t)(2 * box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// K splits of the shared expert's down projection. Its K (= shared intermediate
// size) is several times the routed one, so at decode sizes its few long tiles
// would be the critical path; splitting K yields partial rows that the merge
// sums. Prefill has enough tiles to balance without it.
// Splits are counted in 128-input blocks so both GEMM variants cut K at the
// same places.
int shared_down_parts(int64_t T, int Is) {
  if (Is <= 0) return 0;
  const int kb = Is / 128;
  if (T > 256) return 1;
  for (int parts = 8; parts > 1; --parts)
    if (kb % parts == 0 && kb / parts >= 8) return parts;
  return 1;
}

inline int box_rows_for(int64_t max_rows, int cap) {
  const int64_t r = ((max_rows + 15) / 16) * 16;
  return (int)std::min<int64_t>(cap, std::max<int64_t>(16, r));
}

struct WsLayout {
  size_t h_routed, h_shared, items_gu, items_dn, n_items;
  size_t x8_r, x8_s, h8_r, h8_s, sx_r, sx_s, sh_r, sh_s;
  size_t total;
  int cap_gu, cap_dn;
};

// Work-item capacity is sized for the smaller (64-token) tile cap, which bounds
// both variants; the e4m3 activation planes are laid out for every call.
WsLayout ws_layout(int64_t T, int K, int E, int I, int H, int Is) {
  const int64_t N = T * K;
  const int64_t Isz = Is > 0 ? Is : 0;
  const int64_t tiles_r = N / BN8 + std::min<int64_t>(E, N) + 1;
  const int64_t tiles_s = Is > 0 ? (T + BN8 - 1) / BN8 : 0;
  WsLayout w{};
  w.cap_gu = (int)(tiles_r * (I / BM) + tiles_s * (Is / BM));
  w.cap_dn = (int)((tiles_r + tiles_s * shared_down_parts(T, Is)) * (H / BM));
  size_t o = 0;
  w.h_routed = o; o = align256(o + (size_t)N * I * 2);
  w.h_shared = o; o = align256(o + (size_t)T * Isz * 2);
  w.items_gu = o; o = align256(o + (size_t)w.cap_gu * sizeof(WorkItem));
  w.items_dn = o; o = align256(o + (size_t)w.cap_dn * sizeof(WorkItem));
  w.n_items = o; o = align256(o + 16);
  w.x8_r = o; o = align256(o + (size_t)N * H * 2);
  w.x8_s = o; o = align256(o + (size_t)(Is > 0 ? T : 0) * H * 2);
  w.h8_r = o; o = align256(o + (size_t)N * I * 2);
  w.h8_s = o; o = align256(o + (size_t)T * Isz * 2);
  w.sx_r = o; o = align256(o + (size_t)N * 4);
  w.sx_s = o; o = align256(o + (size_t)T * 4);
  w.sh_r = o; o = align256(o + (size_t)N * 4);
  w.sh_s = o; o = align256(o + (size_t)T * 4);
  w.total = o;
  return w;
}

int g_num_sms = 0;

template <int MODE, int NM, int BNT>
int launch_gemm_f8(const GemmParams& prm, int grid, cudaStream_t stream) {
  using C = Cfg8<MODE, NM, BNT>;
  auto kfn = moe_gemm_f8_kernel<MODE, NM, BNT>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return DWDP_ERR_CUDA;
  return launch_chained(kfn, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, stream, 1u, prm) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

// One warp per row once the rows fill every SM's warps; below that a CTA per
// row (decode: a few long rows want more loads in flight than one warp has).
constexpr int64_t kQuantWarpRows = 148 * 8;
inline int quant_per_warp(int64_t rows) { return rows >= kQuantWarpRows ? 1 : 0; }
inline int quant_blocks(int64_t rows) {
  const int64_t b = quant_per_warp(rows) ? (rows + kPlanThreads / 32 - 1) / (kPlanThreads / 32) : rows;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16));
}

template <int MODE, bool WFP8>
int launch_gemm(const GemmParams& prm, int grid, cudaStream_t stream) {
  using C = Cfg<MODE, WFP8>;
  auto kfn = moe_gemm_kernel<MODE, WFP8>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return DWDP_ERR_CUDA;
  return launch_chained(kfn, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, stream, 1u, prm) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

}  // namespace

extern "C" int dwdp_device_sm_count(void) {
  if (g_num_sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  }
  return g_num_sms;
}

extern "C" int dwdp_moe_shared_parts(int64_t num_tokens, int shared_intermediate_size) {
  return shared_down_parts(num_tokens, shared_intermediate_size);
}

extern "C" size_t dwdp_moe_workspace_bytes_impl(int64_t T, int K, int E, int H, int I, int Is) {
  return ws_layout(T, K, E, I, H, Is).total;
}

// The shared expert alone runs as the launch above with the shared group standing in
// for the routed one (K = 1, E = 1) and no routed rows.
extern "C" size_t dwdp_moe_shared_workspace_bytes_impl(int64_t T, int H, int Is) {
  return ws_layout(T, 1, 1, Is, H, Is).total;
}

extern "C" int dwdp_gather_rows_launch(const void* hidden, const int64_t* tok, int64_t N, int H, int64_t T,
                                       void* packed, int* status, cudaStream_t stream);

// packed_hidden == nullptr: routed row d is hidden[packed_tok[d]] (the e4m3 path
// quantises straight from hidden; the bf16 path gathers into the workspace).
extern "C" int dwdp_moe_experts_launch(const dwdp_expert_group* routed, const dwdp_expert_group* shared,
                                       const void* packed_hidden, const int64_t* packed_tok,
                                       const void* hidden, int64_t T,
                                       int K, const int64_t* counts, const int64_t* offsets,
                                       const float* packed_weights, const float* shared_gate,
                                       void* weighted_out, void* shared_out, void* workspace,
                                       size_t workspace_bytes, int* status, int shared_only,
                                       cudaStream_t stream) {
  // shared_only: the shared expert alone (routed describes its shape; no routed rows)
  if (routed == nullptr || T < 0 || K <= 0) return DWDP_ERR_INVALID_ARGUMENT;
  const int H = routed->hidden_size, I = routed->intermediate_size, E = routed->num_experts;
  const int Is = shared ? shared->intermediate_size : 0;
  if (H % 128 || I % 128 || Is % 128 || E <= 0 || E > 1024) return DWDP_ERR_INVALID_ARGUMENT;
  const bool fp8 = routed->weight_dtype == DWDP_DTYPE_FP8_E4M3;
  if (!fp8 && routed->weight_dtype != DWDP_DTYPE_BF16) return DWDP_ERR_UNSUPPORTED;
  if (shared != nullptr &&
      (shared->weight_dtype != routed->weight_dtype || shared->scale_mode != routed->scale_mode))
    return DWDP_ERR_UNSUPPORTED;  // both groups share one tile layout per launch
  // per-channel e4m3 weights run on the e4m3 tensor-core kernels; block-scaled
  // e4m3 and bf16 weights on the bf16 kernels
  const bool native = fp8 && routed->scale_mode == DWDP_SCALE_CHANNEL;
  const int bk = native ? BK8 : BK;
  // e4m3 token tiles: 64 tokens. 128-token tiles (half the weight traffic per FLOP, one TMEM
  // accumulator buffer for gate/up, 3-deep ring) measured slower at T = 1024 and 4096 on the
  // Qwen shape; DWDP_WIDE_TILES=1 selects them for tuning.
  bool wide = false;
  if (const char* v = getenv("DWDP_WIDE_TILES")) wide = native && v[0] == '1';  // tuning override
  const int bn = native ? (wide ? 128 : BN8) : BN_MAX;
  const int64_t N = shared_only ? 0 : T * K;  // routed rows
  const WsLayout L = ws_layout(T, K, E, I, H, Is);
  if (workspace == nullptr || workspace_bytes < L.total) return DWDP_ERR_CAPACITY;
  if (T == 0) return DWDP_OK;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  __nv_bfloat16* h_r = reinterpret_cast<__nv_bfloat16*>(ws + L.h_routed);
  __nv_bfloat16* h_s = reinterpret_cast<__nv_bfloat16*>(ws + L.h_shared);
  WorkItem* items_gu = reinterpret_cast<WorkItem*>(ws + L.items_gu);
  WorkItem* items_dn = reinterpret_cast<WorkItem*>(ws + L.items_dn);
  int* n_items = reinterpret_cast<int*>(ws + L.n_items);
  float* sx_r = reinterpret_cast<float*>(ws + L.sx_r);
  float* sx_s = reinterpret_cast<float*>(ws + L.sx_s);
  float* sh_r = reinterpret_cast<float*>(ws + L.sh_r);
  float* sh_s = reinterpret_cast<float*>(ws + L.sh_s);
  DeviceStatus* st = reinterpret_cast<DeviceStatus*>(status);
  const int has_shared = shared != nullptr ? 1 : 0;

  const int parts = shared_down_parts(T, Is);
  PlanParams pp{};
  pp.counts = shared_only ? nullptr : counts; pp.offsets = offsets; pp.E = E; pp.T = (int)T;
  pp.has_shared = has_shared;
  // e4m3 path at prefill sizes: a down item covers two consecutive 128-row blocks (one activation
  // tile for two MMAs, half the activation traffic per FLOP). Decode keeps single blocks: there
  // the halved item count would leave SMs idle or unevenly loaded (pairs need ~4 waves of items).
  const int sms_now = dwdp_device_sm_count();
  const int64_t est_tiles = N / BN8 + std::min<int64_t>(E, N) + (has_shared ? (T + BN8 - 1) / BN8 * parts : 0);
  bool pair_dn = native && est_tiles * ((H / BM + 1) / 2) >= 4LL * std::max(1, sms_now);
  if (const char* v = getenv("DWDP_PAIR_DOWN")) pair_dn = native && v[0] == '1';  // tuning override
  const int dn_items_per_tile = pair_dn ? (H / BM + 1) / 2 : H / BM;
  pp.rb_gu_r = I / BM; pp.rb_dn_r = dn_items_per_tile;
  pp.rb_gu_s = has_shared ? Is / BM : 0; pp.rb_dn_s = has_shared ? dn_items_per_tile : 0;
  pp.dn_pair = pair_dn ? 1 : 0; pp.blocks_dn = H / BM;
  pp.kb_gu = H / bk; pp.kb_dn_r = I / bk; pp.kb_dn_s = has_shared ? Is / bk : 0;
  pp.sdn_parts = has_shared ? parts : 0;
  pp.bn_max = bn;
  const long long esz = fp8 ? 1 : 2;
  pp.w_gu[0] = routed->w13; pp.w_dn[0] = routed->w2; pp.s_gu[0] = routed->s13; pp.s_dn[0] = routed->s2;
  pp.rbb_gu[0] = 128LL * H * 2 * esz; pp.rbb_dn[0] = 128LL * I * esz;
  if (has_shared) {
    pp.w_gu[1] = shared->w13; pp.w_dn[1] = shared->w2; pp.s_gu[1] = shared->s13; pp.s_dn[1] = shared->s2;
    pp.rbb_gu[1] = 128LL * H * 2 * esz; pp.rbb_dn[1] = 128LL * Is * esz;
  }
  pp.items_gu = items_gu; pp.items_dn = items_dn; pp.n_items = n_items;
  pp.cap_gu = L.cap_gu; pp.cap_dn = L.cap_dn; pp.st = st;
  QuantParams qx{}, qh{};
  qx.st = st;
  qh.st = st;
  qx.per_warp = qh.per_warp = quant_per_warp(N + (has_shared ? T : 0));
  const bool indexed = packed_hidden == nullptr;
  if (indexed && packed_tok == nullptr && N > 0) return DWDP_ERR_INVALID_ARGUMENT;
  if (native) {
    const __nv_bfloat16* hid = reinterpret_cast<const __nv_bfloat16*>(hidden);
    qx.seg[0] = indexed ? QuantSeg{hid, ws + L.x8_r, sx_r, (int)N, H, packed_tok, T}
                        : QuantSeg{reinterpret_cast<const __nv_bfloat16*>(packed_hidden), ws + L.x8_r, sx_r,
                                   (int)N, H, nullptr, N};
    if (has_shared) qx.seg[1] = QuantSeg{hid, ws + L.x8_s, sx_s, (int)T, H, nullptr, T};
    qh.seg[0] = QuantSeg{h_r, ws + L.h8_r, sh_r, (int)N, I, nullptr, N};
    if (has_shared) qh.seg[1] = QuantSeg{h_s, ws + L.h8_s, sh_s, (int)T, Is, nullptr, T};
  } else if (indexed && N > 0) {
    // the bf16 kernels stream packed rows by TMA: gather them into the (unused) plane area
    const int rc = dwdp_gather_rows_launch(hidden, packed_tok, N, H, T, ws + L.x8_r, status, stream);
    if (rc != DWDP_OK) return rc;
    packed_hidden = ws + L.x8_r;
  }
  const int qx_blocks = native ? quant_blocks(N + (has_shared ? T : 0)) : 0;
  if (launch_chained(prep_kernel, dim3(kPlanBlocks + qx_blocks), dim3(kPlanThreads), 0, stream, 1u, pp, qx) !=
      cudaSuccess)
    return DWDP_ERR_CUDA;

  // The activation box must cover the largest tile: a routed tile holds at most
  // min(T * K, bn) rows (an expert may be picked more than once per token), a
  // shared tile at most min(T, bn).
  const int box_r = box_rows_for(N, bn), box_s = box_rows_for(T, bn);
  auto map = [&](CUtensorMap* m, const void* bf16, size_t planes_off, int64_t rows, int64_t cols, int box) {
    return native ? make_tmap_planes(m, ws + planes_off, rows, cols, box) : make_tmap(m, bf16, rows, cols, box);
  };
  GemmParams gu{}, dn{};
  gu.g[0].enabled = N > 0;
  if (N > 0 && !map(&gu.g[0].tmap_b, packed_hidden, L.x8_r, N, H, box_r)) return DWDP_ERR_CUDA;
  gu.g[0].w = routed->w13; gu.g[0].s = routed->s13; gu.g[0].out = h_r; gu.g[0].row_scale = nullptr;
  gu.g[0].x_scale = sx_r;
  gu.g[0].K = H; gu.g[0].R = I; gu.g[0].scale_mode = routed->scale_mode; gu.g[0].box_rows = box_r;
  // e4m3 tiles: gate/up interleaved per 128-input stage; down row blocks are K/128 tiles apart
  gu.g[0].mstride = kW8TileBytes; gu.g[0].kstride = 2 * kW8TileBytes;
  gu.g[1].enabled = has_shared;
  if (has_shared) {
    if (!map(&gu.g[1].tmap_b, hidden, L.x8_s, T, H, box_s)) return DWDP_ERR_CUDA;
    gu.g[1].w = shared->w13; gu.g[1].s = shared->s13; gu.g[1].out = h_s; gu.g[1].row_scale = nullptr;
    gu.g[1].x_scale = sx_s;
    gu.g[1].K = H; gu.g[1].R = Is; gu.g[1].scale_mode = shared->scale_mode; gu.g[1].box_rows = box_s;
    gu.g[1].mstride = kW8TileBytes; gu.g[1].kstride = 2 * kW8TileBytes;
  }
  gu.items = items_gu; gu.n_items = n_items; gu.st = st; gu.cap = L.cap_gu;

  dn.g[0].enabled = N > 0;
  if (N > 0 && !map(&dn.g[0].tmap_b, h_r, L.h8_r, N, I, box_r)) return DWDP_ERR_CUDA;
  dn.g[0].w = routed->w2; dn.g[0].s = routed->s2; dn.g[0].out = weighted_out; dn.g[0].box_rows = box_r;
  dn.g[0].x_scale = sh_r;
  dn.g[0].row_scale = packed_weights; dn.g[0].K = I; dn.g[0].R = H; dn.g[0].scale_mode = routed->scale_mode;
  dn.g[0].mstride = (long long)BM * I; dn.g[0].kstride = kW8TileBytes;
  dn.g[1].enabled = has_shared;
  if (has_shared) {
    if (!map(&dn.g[1].tmap_b, h_s, L.h8_s, T, Is, box_s)) return DWDP_ERR_CUDA;
    dn.g[1].w = shared->w2; dn.g[1].s = shared->s2; dn.g[1].out = shared_out; dn.g[1].box_rows = box_s;
    dn.g[1].x_scale = sh_s;
    dn.g[1].row_scale = shared_gate; dn.g[1].K = Is; dn.g[1].R = H; dn.g[1].scale_mode = shared->scale_mode;
    dn.g[1].mstride = (long long)BM * Is; dn.g[1].kstride = kW8TileBytes;
    dn.g[1].part_stride = (long long)T * H;
  }
  dn.items = items_dn; dn.n_items = n_items + 1; dn.st = st; dn.cap = L.cap_dn;

  const int sms = dwdp_device_sm_count();
  if (sms <= 0) return DWDP_ERR_CUDA;
  const int grid_gu = std::max(1, std::min(sms, L.cap_gu));
  const int grid_dn = std::max(1, std::min(sms, L.cap_dn));
  int rc;
  if (native) {
    rc = wide ? launch_gemm_f8<0, 2, 128>(gu, grid_gu, stream) : launch_gemm_f8<0, 2, 64>(gu, grid_gu, stream);
    if (rc == DWDP_OK) {
      rc = launch_chained(quant_kernel, dim3(quant_blocks(N + (has_shared ? T : 0))), dim3(kPlanThreads), 0,
                          stream, 1u, qh) == cudaSuccess
               ? DWDP_OK
               : DWDP_ERR_CUDA;
    }
    if (rc == DWDP_OK) {
      if (wide) rc = pair_dn ? launch_gemm_f8<1, 2, 128>(dn, grid_dn, stream) : launch_gemm_f8<1, 1, 128>(dn, grid_dn, stream);
      else rc = pair_dn ? launch_gemm_f8<1, 2, 64>(dn, grid_dn, stream) : launch_gemm_f8<1, 1, 64>(dn, grid_dn, stream);
    }
  } else if (fp8) {
    rc = launch_gemm<0, true>(gu, grid_gu, stream);
    if (rc == DWDP_OK) rc = launch_gemm<1, true>(dn, grid_dn, stream);
  } else {
    rc = launch_gemm<0, false>(gu, grid_gu, stream);
    if (rc == DWDP_OK) rc = launch_gemm<1, false>(dn, grid_dn, stream);
  }
  return rc;
}

#ifdef DWDP_PROFILE_ROLES
extern "C" int dwdp_debug_role_cycles(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, dwdp::g_role_cycles, sizeof(dwdp::g_role_cycles)) == cudaSuccess ? 0 : -3;
}
#endif

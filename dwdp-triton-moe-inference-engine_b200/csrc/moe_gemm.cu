// Grouped expert GEMMs on tcgen05 (sm_100a): the executor hot path.
//
// Replaces the per-expert loop of DWDP/executor/pytorch.py:66-160 (gather,
// down(silu(gate(x)) * up(x)), times routing weight), the Triton persistent
// kernels of DWDP/executor/kernels/persistent.py:241-401 / fp8.py:147-318 and the
// block-scaled FP8 executor of DWDP/executor/triton_tma.py:115-261.
//
// Orientation ("swap AB"): the weight rows of one 128-row block are the MMA M
// dimension (TMEM lanes), the tokens of one expert tile are the MMA N dimension
// (16..128 columns, chosen per expert so a 273-row expert runs as 3 x 96, not
// 3 x 128). A per-output-channel or per-block weight scale therefore becomes a
// per-thread constant, and a decode step with one token per expert still fills
// the 128-row MMA with weights.
//
// Two GEMM launches per layer, after a planning launch:
//   MODE 0  gate/up: acc_g, acc_u [128 feat x N tok] in TMEM (two MMAs sharing
//           the activation tile), epilogue h = silu(g) * u
//   MODE 1  down   : acc [128 out x N tok], epilogue y * row_scale -> bf16 out
//
// Three kernel families (warp 0 producer, warp 1 TMEM allocator + single-thread
// MMA issuer, the rest epilogue; one CTA per SM, persistent over a device-built
// work list):
//   moe_gemm_kernel      bf16 weights, kind::f16 MMAs on bf16 activations.
//   moe_gemm_f8_kernel   e4m3 weights with per-row (channel / tensor) scales and
//                        hi/lo e4m3 activation planes (DWDP_ACT_HILO): kind::f8f6f4
//                        MMAs, scales applied once in the epilogue.
//   moe_gemm_f8p_kernel  e4m3 weights of any scale mode against activations whose
//                        scale changes every 128 inputs (DWDP_ACT_BLOCK128, or
//                        128x128 block-scaled weights): every 128-wide K block
//                        accumulates into its own TMEM slot and the epilogue warps
//                        promote it into fp32 registers with its scales.
// and two CTA-pair kernels (tcgen05 cta_group::2, clusters of two CTAs sharing one
// 256 x 256 MMA, orientation tokens x features) for prefill-sized batches:
//   moe_gemm_f8x2_kernel   hi/lo activation planes, per-row weight scales.
//   moe_gemm_f8x2p_kernel  one activation plane per (row, 128) (DWDP_ACT_BLOCK128),
//                          any weight scale mode, per-K-block promotion.
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
constexpr int kBf16TileBytes = BM * 128;   // bf16 weight tile 128 x 64

struct WorkItem {
  int group;     // 0 routed, 1 shared
  int expert;    // expert index inside the group
  int rb;        // 128-row weight block
  int row0;      // first activation row of the tile
  int nrows;     // rows in this tile (<= BN_MAX)
  int kb_begin;  // first / one-past-last K step of this item (split K)
  int kb_end;
  int part;      // K-split index: output goes to out + part * part_stride
  int nmat;      // weight matrices of the item: gate+up (2), or 1-2 consecutive down row blocks
  const uint8_t* wtiles;  // first weight tile of this item's 128-row block (set by the planner)
  const float* scales;    // the expert's scales (fp8) or nullptr
};

struct GroupParams {
  CUtensorMap tmap_b;      // activations (bf16 rows, hi/lo planes or one e4m3 plane)
  const void* const* w;    // [E] packed weight tiles
  const float* const* s;   // [E] scales (fp8) or nullptr
  void* out;               // bf16 [rows, R]; e4m3 [rows, R] for the BLOCK128 gate/up epilogue
  float* out_scale;        // BLOCK128 gate/up: scales of `out`, [R / 128][os_ld]
  const float* row_scale;  // MODE 1: per-row multiplier (routing weight / shared gate) or null
  const float* x_scale;    // hi/lo: per-row activation scale; BLOCK128: [K / 128][xs_ld]
  int K;                   // reduction size
  int R;                   // output rows of the projection (= out leading dim)
  int scale_mode;
  int enabled;
  int box_rows;            // activation rows per TMA box (multiple of 16, <= BN_MAX)
  long long part_stride;   // elements between K-split partial outputs
  long long mstride;       // e4m3 path: bytes between an item's weight matrices
  long long kstride;       // e4m3 path: bytes between an item's 128-input stages
  long long xs_ld;         // BLOCK128: leading dimension of x_scale (activation rows)
  long long os_ld;         // BLOCK128: leading dimension of out_scale
};

struct GemmParams {
  GroupParams g[2];
  const WorkItem* items;
  const int* n_items;
  int cap;  // work-item capacity (grid <= cap, so items[blockIdx.x] is always addressable)
  DeviceStatus* st;
};

__host__ __device__ inline bool per_row_scales(int mode) {
  return mode == DWDP_SCALE_CHANNEL || mode == DWDP_SCALE_TENSOR;
}

template <int MODE>
struct Cfg {
  static constexpr int NMAT = MODE == 0 ? 2 : 1;
  static constexpr int S = MODE == 0 ? 4 : 6;  // load stages
  static constexpr int W_STAGE_BYTES = NMAT * kBf16TileBytes;
  static constexpr int NUM_WARPS = 6;
  static constexpr int THREADS = NUM_WARPS * 32;
  static constexpr int TMEM_COLS = NMAT * BN_MAX * 2 <= 256 ? 256 : 512;
  static constexpr int ACC_STRIDE = NMAT * BN_MAX;  // TMEM columns per accumulator buffer
  static constexpr int SMEM_B = S * kBTileBytes;
  static constexpr int SMEM_W = S * W_STAGE_BYTES;
  static constexpr int SMEM_BYTES = SMEM_B + SMEM_W + 1024 /*align*/ + 256 /*barriers*/;
};

// bf16 weights: kind::f16 MMAs on bf16 activation rows (TMA box {64, BN_MAX}).
template <int MODE>
__global__ void __launch_bounds__(Cfg<MODE>::THREADS, 1)
moe_gemm_kernel(const __grid_constant__ GemmParams p) {
  using C = Cfg<MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sW = sB + C::SMEM_B;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + C::SMEM_W);
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
      uint32_t it = 0;
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
          tc_fence_after();
          // Descriptors are built once per stage; a K step of 16 bf16 (32 bytes) is +2 in
          // the encoded start address, the second weight matrix is +kBf16TileBytes/16.
          const uint64_t b_desc0 = smem_desc_sw128(smem_u32(sB + s * kBTileBytes));
          const uint64_t a_desc0 = smem_desc_sw128(smem_u32(sW + s * C::W_STAGE_BYTES));
          const uint32_t acc_first = kb > wi.kb_begin ? 1u : 0u;
          PROF_T0
#pragma unroll
          for (int m = 0; m < C::NMAT; ++m) {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              mma_bf16_ss(d_base + m * BN_MAX, a_desc0 + (uint64_t)(m * (kBf16TileBytes >> 4) + 2 * kk),
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
              const float h = silu(gv[j]) * uv[j];
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
              out[(size_t)row * g.R + feat] = __float2bfloat16_rn(yv[j] * sc);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
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
// CTA-pair (cta_group::2) primitives for moe_gemm_f8x2_kernel. Every tcgen05
// instruction of that kernel uses cta_group::2; none issues a multicast load.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on the mbarrier at the same shared-memory offset in CTA `cta` of the cluster. The
// waiter polls with the usual CTA-scope acquire (as for any barrier): the data the phase
// announces is read by the tensor core through the async proxy, not by the waiting thread.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, uint32_t cta) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
      "r"(cta)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A * B^T over the CTA pair: A = 128 rows in each CTA's shared memory
// (M = 256), B = N / 2 rows in each CTA's shared memory, same offsets in both CTAs.
__device__ __forceinline__ void mma2_e4m3_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// Arrive once on the mbarrier at the same offset in every CTA of `mask` when the pair's
// previously issued MMAs complete.
__device__ __forceinline__ void mma2_commit_mc(uint64_t* bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"(mask)
               : "memory");
}

// ---------------------------------------------------------------------------
// e4m3 hi/lo GEMMs on a CTA pair (cta_group::2), for prefill-sized batches.
//
// A single CTA feeds 48 KB per 128-input stage (two 16 KB weight tiles + a 16 KB
// hi/lo activation tile for 64 tokens); with the MMAs running, an SM's bulk-copy
// fill rate caps that at ~840 cycles per stage against the MMAs' 512. Here two
// SMs share one 256 x 256 MMA per 32 inputs, orientation tokens x features:
//   A (M = 256): the activation planes of up to 128 tokens, 64 per CTA (rows
//                2t = hi, 2t + 1 = lo of token t), 16 KB per CTA per stage;
//   B (N = 256): MODE 0 gate rows (CTA 0) | up rows (CTA 1) of one 128-feature
//                block; MODE 1 two consecutive 128-row down blocks; 16 KB per CTA.
// So each SM moves 32 KB per stage for the same MMA work, and a 7-deep ring fits.
// Each CTA's TMEM holds its 128 plane rows x 256 columns (double-buffered). The
// leader (rank 0) issues the MMAs once both CTAs' stage is loaded (the peer's
// MMA-issue thread relays its local barrier phases to the leader) and its
// commits arrive on both CTAs' barriers. Epilogue: lane pairs (hi, lo) swap
// halves so every lane forms 16 features of one token, then 32-byte stores.
// ---------------------------------------------------------------------------
#ifndef DWDP_X2_DIAG
#define DWDP_X2_DIAG 0  // diagnostic builds only: 1 = no epilogue math (wrong results, timing only)
#endif
// KPS = 128-input K blocks per pipeline stage: 2 halves the number of copies (one 3-D TMA box
// for both activation tiles, one bulk copy for both weight tiles where they are contiguous).
template <int MODE, int KPS>
struct CfgX2 {
  static constexpr int A_TILE = 128 * BK8;  // 64 tokens x 2 planes x 128 inputs
  static constexpr int B_TILE = kW8TileBytes;  // 128 weight rows x 128 inputs
  static constexpr int STAGE_A = KPS * A_TILE;
  static constexpr int STAGE_B = KPS * B_TILE;
  static constexpr int STAGE = STAGE_A + STAGE_B;
  static constexpr int S = KPS == 1 ? 7 : 3;
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int THREADS = (2 + EPI_WARPS) * 32;
  static constexpr int ACC_COLS = 256;
  static constexpr int SMEM_BYTES = S * STAGE + 1024 + 512;
};

template <int MODE, int KPS>
__global__ void __launch_bounds__(CfgX2<MODE, KPS>::THREADS, 1) moe_gemm_f8x2_kernel(const __grid_constant__ GemmParams p) {
  using C = CfgX2<MODE, KPS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::S * C::STAGE_A;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::S * C::STAGE);
  uint64_t* full = bars;               // local loads of stage s landed
  uint64_t* empty = full + C::S;       // the pair's MMAs read stage s (leader commit, both CTAs)
  uint64_t* peer_full = empty + C::S;  // leader only: the peer's stage s landed
  uint64_t* acc_full = peer_full + C::S;  // accumulator a ready (leader commit, both CTAs)
  uint64_t* acc_empty = acc_full + 2;     // this CTA's epilogue drained accumulator a
  uint64_t* peer_acc_empty = acc_empty + 2;  // leader only: the peer's epilogue drained a
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_rank();
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  DeviceStatus* st = p.st;
  griddep_launch();
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < C::S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&peer_full[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], C::EPI_THREADS);
      mbar_init(&peer_acc_empty[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc2(&s_tmem_base, 2 * C::ACC_COLS);
    tmem_relinquish2();
  }
  if (warp == 0 && lane == 0) {
    if (p.g[0].enabled) prefetch_tmap(&p.g[0].tmap_b);
    if (p.g[1].enabled) prefetch_tmap(&p.g[1].tmap_b);
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = s_tmem_base;
  griddep_wait();
  const int n_items = *p.n_items;
  if (warp == 0) {
    // ------------------------------------------------------------ producer (each CTA its halves)
    if (lane == 0) {
      PROF_DECL PROF_START
      uint32_t it = 0;
      for (int item = cid; item < n_items && !s_abort; item += ncl) {
        const WorkItem wi = p.items[item];
        const GroupParams& g = p.g[wi.group];
        const int h = min(64, (wi.nrows + 1) >> 1);  // tokens of CTA 0; CTA 1 takes the rest
        const int tok0 = wi.row0 + (int)rank * h;
        const uint8_t* wsrc = wi.wtiles + (size_t)rank * g.mstride;
        for (int kb = wi.kb_begin; kb < wi.kb_end; kb += KPS, ++it) {
          const int s = it % C::S;
          const int nkb = min(KPS, wi.kb_end - kb);
          if (!TW(0, mbar_wait(&empty[s], ((it / C::S) & 1) ^ 1, &s_abort, st, 61 + 8 * MODE))) break;
          // the activation box always lands whole (K blocks past the end read as zeros)
          mbar_arrive_expect_tx(&full[s], (uint32_t)(C::STAGE_A + nkb * C::B_TILE));
          if (g.kstride == C::B_TILE) {
            bulk_g2s(sB + s * C::STAGE_B, wsrc + (size_t)kb * g.kstride, nkb * C::B_TILE, &full[s]);
          } else {
            for (int q = 0; q < nkb; ++q)
              bulk_g2s(sB + s * C::STAGE_B + q * C::B_TILE, wsrc + (size_t)(kb + q) * g.kstride, C::B_TILE, &full[s]);
          }
          if constexpr (KPS == 1) tma_load_2d(sA + s * C::STAGE_A, &g.tmap_b, kb * BK8, 2 * tok0, &full[s]);
          else tma_load_3d(sA + s * C::STAGE_A, &g.tmap_b, 0, 2 * tok0, kb, &full[s]);
        }
      }
      PROF_END(7) PROF_STORE(0)
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------------ MMA issuer (leader)
      PROF_DECL PROF_START
      uint32_t it = 0;
      int li = 0;
      const uint32_t idesc = idesc_e4m3(256, 256);
      for (int item = cid; item < n_items && !s_abort; item += ncl, ++li) {
        const WorkItem wi = p.items[item];
        const int a = li & 1;
        const uint32_t par = ((li >> 1) & 1) ^ 1;
        if (!TW(0, mbar_wait(&acc_empty[a], par, &s_abort, st, 62 + 8 * MODE))) break;
        if (!TW(1, mbar_wait(&peer_acc_empty[a], par, &s_abort, st, 63 + 8 * MODE))) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * C::ACC_COLS;
        bool ok = true;
        for (int kb = wi.kb_begin; kb < wi.kb_end; kb += KPS, ++it) {
          const int s = it % C::S;
          const int nkb = min(KPS, wi.kb_end - kb);
          const uint32_t fp = (it / C::S) & 1;
          if (!TW(2, mbar_wait(&full[s], fp, &s_abort, st, 64 + 8 * MODE)) ||
              !TW(3, mbar_wait(&peer_full[s], fp, &s_abort, st, 65 + 8 * MODE))) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int q = 0; q < nkb; ++q) {
            const uint64_t ad = smem_desc_sw128(smem_u32(sA + s * C::STAGE_A + q * C::A_TILE));
            const uint64_t bd = smem_desc_sw128(smem_u32(sB + s * C::STAGE_B + q * C::B_TILE));
#pragma unroll
            for (int kk = 0; kk < BK8 / 32; ++kk)
              mma2_e4m3_ss(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), idesc,
                           (kk > 0 || q > 0 || kb > wi.kb_begin) ? 1u : 0u);
          }
          mma2_commit_mc(&empty[s], 0x3);
        }
        if (!ok) break;
        mma2_commit_mc(&acc_full[a], 0x3);
      }
      PROF_END(7) PROF_STORE(4)
    } else if (lane == 0) {
      // ------------------------------------------------------------ relay (peer): local phases -> leader
      PROF_DECL PROF_START
      uint32_t it = 0;
      int li = 0;
      for (int item = cid; item < n_items && !s_abort; item += ncl, ++li) {
        const WorkItem wi = p.items[item];
        const int a = li & 1;
        if (li >= 2) {
          if (!TW(0, mbar_wait(&acc_empty[a], ((li >> 1) & 1) ^ 1, &s_abort, st, 66 + 8 * MODE))) break;
          mbar_arrive_remote(&peer_acc_empty[a], 0);
        }
        bool ok = true;
        for (int kb = wi.kb_begin; kb < wi.kb_end; kb += KPS, ++it) {
          const int s = it % C::S;
          if (!TW(1, mbar_wait(&full[s], (it / C::S) & 1, &s_abort, st, 67 + 8 * MODE))) {
            ok = false;
            break;
          }
          mbar_arrive_remote(&peer_full[s], 0);
        }
        if (!ok) break;
      }
      PROF_END(7) PROF_STORE(4)
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;              // TMEM lanes 32 quad .. 32 quad + 31
    const int hw = (warp - 2) >> 2;         // column half of the item this warp drains
    const int t_loc = quad * 16 + (lane >> 1);  // token of this lane inside the CTA's 64
    const int odd = lane & 1;               // 0: hi row, keeps columns 0-15 of a chunk; 1: lo, 16-31
    PROF_DECL PROF_START
    int li = 0;
    for (int item = cid; item < n_items; item += ncl, ++li) {
      if (__any_sync(0xffffffffu, s_abort != 0)) break;  // warp-uniform exit (the warp shuffles below)
      const WorkItem wi = p.items[item];
      const GroupParams& g = p.g[wi.group];
      const int a = li & 1;
      const int h = min(64, (wi.nrows + 1) >> 1);
      const int n_my = rank == 0 ? h : wi.nrows - h;
      const int tok = wi.row0 + (int)rank * h + t_loc;
      const bool live = t_loc < n_my;
      float fx = 0.f;
      if (live) {
        fx = g.x_scale[tok];
        if (MODE == 1 && g.row_scale != nullptr) fx *= g.row_scale[tok];
      }
      const bool got = TW(0, mbar_wait(&acc_full[a], (li >> 1) & 1, &s_abort, st, 68 + 8 * MODE));
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + a * C::ACC_COLS + ((uint32_t)(quad * 32) << 16);
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)wi.part * g.part_stride;
      // MODE 0: this warp takes gate/up features [64 hw, 64 hw + 64) in two 32-column chunks;
      // MODE 1: output columns [128 hw, 128 hw + 128) in four chunks.
      constexpr int NCH = MODE == 0 ? 2 : 4;
      uint4 res[NCH][2];
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int c0 = (MODE == 0 ? 64 : 128) * hw + 32 * c;  // first column of the chunk
        float v[MODE == 0 ? 2 : 1][32];
        tmem_ld32(t_acc + c0, v[0]);
        if constexpr (MODE == 0) tmem_ld32(t_acc + 128 + c0, v[1]);
        tmem_ld_wait();
        // combine hi + lo / 16 for 16 columns per lane: hi lanes keep 0-15, lo lanes 16-31
        float r[MODE == 0 ? 2 : 1][16];
#pragma unroll
        for (int m = 0; m < (MODE == 0 ? 2 : 1); ++m) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float send = odd ? v[m][k] : v[m][16 + k];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
            r[m][k] = odd ? recv + v[m][16 + k] * (1.0f / kLoPlaneGain) : v[m][k] + recv * (1.0f / kLoPlaneGain);
          }
        }
        const int col = c0 + odd * 16;  // first item column of this lane's 16
        uint32_t packed[8];
        if (DWDP_X2_DIAG & 1) {  // diagnostic build: no epilogue math
          res[c][0] = res[c][1] = make_uint4(__float_as_uint(r[0][0]), 0, 0, 0);
          continue;
        }
        if constexpr (MODE == 0) {
          const int f = wi.rb * BM + col;  // feature of the projection (16-float aligned)
          float sg[16], su[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 a4 = __ldg(reinterpret_cast<const float4*>(wi.scales + f) + q);
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(wi.scales + g.R + f) + q);
            sg[4 * q] = a4.x; sg[4 * q + 1] = a4.y; sg[4 * q + 2] = a4.z; sg[4 * q + 3] = a4.w;
            su[4 * q] = b4.x; su[4 * q + 1] = b4.y; su[4 * q + 2] = b4.z; su[4 * q + 3] = b4.w;
          }
#pragma unroll
          for (int k = 0; k < 16; k += 2) {
            const float g0 = r[0][k] * (sg[k] * fx), g1 = r[0][k + 1] * (sg[k + 1] * fx);
            const float u0 = r[1][k] * (su[k] * fx), u1 = r[1][k + 1] * (su[k + 1] * fx);
            const __nv_bfloat162 hv = __floats2bfloat162_rn(silu_fast(g0) * u0, silu_fast(g1) * u1);
            packed[k >> 1] = *reinterpret_cast<const uint32_t*>(&hv);
          }
        } else {
          const int f = wi.rb * BM + col;  // output feature (two consecutive 128-row blocks)
          float sw[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 a4 = __ldg(reinterpret_cast<const float4*>(wi.scales + f) + q);
            sw[4 * q] = a4.x; sw[4 * q + 1] = a4.y; sw[4 * q + 2] = a4.z; sw[4 * q + 3] = a4.w;
          }
#pragma unroll
          for (int k = 0; k < 16; k += 2) {
            const __nv_bfloat162 yv =
                __floats2bfloat162_rn(r[0][k] * (sw[k] * fx), r[0][k + 1] * (sw[k + 1] * fx));
            packed[k >> 1] = *reinterpret_cast<const uint32_t*>(&yv);
          }
        }
        res[c][0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        res[c][1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);  // the accumulator is drained; stores follow
      if (live && !(DWDP_X2_DIAG & 1)) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int col = (MODE == 0 ? 64 : 128) * hw + 32 * c + odd * 16;
          uint4* dst = reinterpret_cast<uint4*>(out + (size_t)tok * g.R + wi.rb * BM + col);
          dst[0] = res[c][0];
          dst[1] = res[c][1];
        }
      }
    }
    PROF_END(7) if (lane == 0 && warp == 2) PROF_STORE(8)
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // both CTAs done: the leader's MMAs and both epilogues
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, 2 * C::ACC_COLS);
  }
}

// ---------------------------------------------------------------------------
// e4m3 tensor-core path with per-128-K-block promotion.
//
// Used when the product's scale changes along K every 128 inputs: activations
// quantised per (row, 128 channels) (DWDP_ACT_BLOCK128, the reference's FP8
// scheme, DWDP/executor/fp8.py:86-115) and/or weights with 128x128 block scales
// (DWDP/executor/fp8.py:118-146). The reference's kernel applies the scales to
// its fp32 accumulator once per K block (DWDP/executor/kernels/fp8_tma.py:104-119):
//   C = sum_kb (Xq Wq^T)_kb * sx[row, kb] * sw[nb, kb]
// Here every 128-wide K block of an item is multiplied into its own TMEM slot
// (a ring of NSLOT slots, so the tensor core runs up to NSLOT blocks ahead) and
// the epilogue warps fold it into fp32 registers:
//   acc[m][t] += slot[m][t] * (sx[t][kb] * sw[m][kb])
// PLANES = 1: one e4m3 activation plane, one MMA column per token, sx per
//             (row, 128). The gate/up epilogue rounds gate/up to bf16, forms the
//             SwiGLU product in bf16 (as the reference's executor does in its
//             output dtype) and re-quantises it per (row, 128 features) = per
//             row of the item's 128-row weight block, writing the e4m3 rows and
//             their scales for the down projection directly.
// PLANES = 2: hi/lo planes (block-scaled weights in the high-accuracy mode):
//             acc += sw[kb] * (hi + lo / 16), the per-row sx applied at the end.
// Per-row weight scales (CHANNEL / TENSOR) are applied once at the end.
// Epilogue warp (quadrant q = warp % 4, chunk c) owns TMEM lanes 32q..32q+31
// (weight rows) and the item's tokens [c * TOKW, (c + 1) * TOKW).
// ---------------------------------------------------------------------------
template <int MODE, int NM, int BNT, int PLANES>
struct CfgP {
  static constexpr int NMAT = NM;
  static constexpr int NCOL = PLANES * BNT;               // MMA N per weight matrix (largest tile)
  static constexpr int B_TILE = NCOL * BK8;               // activation bytes per stage
  static constexpr int W_STAGE_BYTES = NMAT * kW8TileBytes;
  static constexpr int SLOT = NMAT * NCOL;                // TMEM columns per K-block slot
  static constexpr int NSLOT = 512 / SLOT > 4 ? 4 : 512 / SLOT;
  static constexpr int TMEM_COLS = NSLOT * SLOT <= 256 ? 256 : 512;
  // Tokens per epilogue warp: 32 with one activation plane (eight epilogue warps for 64-token
  // tiles, so each thread has 168 registers and the promoted accumulators never spill: with
  // sixteen warps the 96-register budget spilled them and every K block paid local-memory
  // round trips), 16 with hi/lo planes (two TMEM columns per token).
#ifdef DWDP_TOKW16
  static constexpr int TOKW = 16;
#else
  static constexpr int TOKW = PLANES == 1 ? 32 : 16;
#endif
  static constexpr int TCOL = PLANES * TOKW;               // TMEM columns per warp and matrix
  static constexpr int CHUNKS = BNT / TOKW;
  static constexpr int EPI_WARPS = 4 * CHUNKS;
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int THREADS = (2 + EPI_WARPS) * 32;
  // Registers per thread: each of the SM's four sub-partitions holds 16384 registers and
  // receives every fourth warp, so the fullest one (ceil(warps / 4) warps) sets the limit
  // (8-register granularity); at most 168.
  static constexpr int WARPS = THREADS / 32;
  static constexpr int REG_FIT = 16384 / (((WARPS + 3) / 4) * 32) / 8 * 8;
  static constexpr int MAXREG = REG_FIT > 168 ? 168 : REG_FIT;
  // every matrix's TMEM columns of a K block loaded at once when accumulators + loaded columns
  // leave ~40 registers for the rest; else 16 columns at a time
  static constexpr bool ALL_AT_ONCE = NMAT * (TOKW + TCOL) + 40 <= MAXREG;
  static constexpr bool QOUT = MODE == 0 && PLANES == 1;   // gate/up writes e4m3 rows + scales
  static constexpr int STAGING = QOUT ? BNT * BM : 0;      // e4m3 [tokens][128 features]
  // per-warp ring of K-block scales, filled DIST blocks ahead with asynchronous copies. A slot
  // holds [32 token scales | 4: NMAT weight-block scales | NMAT x 32 promotion factors]: with
  // one activation plane and block-scaled weights each lane writes its token's factor
  // s_x[t] * s_w[m] once per K block, so the promotion is one FMA per element (every slot
  // starts on a 16-byte boundary: the factors are read as float4).
  static constexpr int FAC = 36;                            // offset of the factors in a slot
  static constexpr int RING = 4, DIST = 3, RSTRIDE = PLANES == 1 ? FAC + NMAT * 32 : 36;
  static_assert(RSTRIDE % 4 == 0, "ring slots must stay 16-byte aligned");
  static_assert(NMAT <= RSTRIDE - 32, "weight-block scales must fit the slot padding");
  static constexpr int SCL = EPI_WARPS * RING * RSTRIDE * 4;
  static constexpr int RED = QOUT ? 4 * BNT * 4 : 0;       // per-quadrant token amax
  static constexpr int FIXED = STAGING + SCL + RED + 1024 /*align*/ + 512 /*barriers*/;
  static constexpr int S = (227 * 1024 - FIXED) / (W_STAGE_BYTES + B_TILE);
  static constexpr int SMEM_BYTES = S * (W_STAGE_BYTES + B_TILE) + FIXED;
  static_assert(S >= 2, "pipeline too shallow");
  static_assert(NSLOT >= 2, "need at least two TMEM slots");
};

#ifdef DWDP_PROFILE_ROLES
// Diagnostic build only: cycles each role of moe_gemm_f8p_kernel spends per activity, in
// g_role_cycles[cta][32 * MODE + slot] (producer 0-1, MMA issuer 2-4, epilogue warp 2: 5-10).
#define RP_TIMED(slot, call) ([&]() { const long long t_ = clock64(); const bool r_ = (call); \
    rp_[slot] += (unsigned long long)(clock64() - t_); return r_; }())
#define RP_BEGIN unsigned long long rp_[16] = {}; const long long rp0_ = clock64();
#define RP_MARK long long rpm_ = clock64();
#define RP_ADD(slot) { const long long n_ = clock64(); rp_[slot] += (unsigned long long)(n_ - rpm_); rpm_ = n_; }
#define RP_END(total, lo, hi) { rp_[total] = (unsigned long long)(clock64() - rp0_); \
    for (int q_ = lo; q_ <= hi; ++q_) g_role_cycles[blockIdx.x][32 * MODE + q_] = rp_[q_]; }
#else
#define RP_TIMED(slot, call) (call)
#define RP_BEGIN
#define RP_MARK
#define RP_ADD(slot)
#define RP_END(total, lo, hi)
#endif

// The f8p kernel's pipeline waits park the waiting thread in hardware (DWDP_SPIN_WAITS: poll).
#ifdef DWDP_SPIN_WAITS
#define MBAR_WAIT_P mbar_wait
#else
#define MBAR_WAIT_P mbar_wait_backoff
#endif

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// (a0, a1) += (v0, v1) * (f0, f1) as one packed fp32x2 FMA (round to nearest).
__device__ __forceinline__ void ffma2(float& a0, float& a1, float v0, float v1, float f0, float f1) {
  asm("{\n\t.reg .b64 va, vf, vc;\n\t"
      "mov.b64 va, {%2, %3};\n\t"
      "mov.b64 vf, {%4, %5};\n\t"
      "mov.b64 vc, {%0, %1};\n\t"
      "fma.rn.f32x2 vc, va, vf, vc;\n\t"
      "mov.b64 {%0, %1}, vc;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(v0), "f"(v1), "f"(f0), "f"(f1));
}

// acc += v * f for a pair of tokens: one packed fp32x2 FMA (measured 4 % faster on the
// gate/up promotion than two scalar FMAs); DWDP_SCALAR_FMA builds the scalar pair.
__device__ __forceinline__ void fma_pair(float& a0, float& a1, float v0, float v1, float f0, float f1) {
#if defined(DWDP_DIAG_NO_FMA)
  a0 += v0; (void)a1; (void)v1; (void)f0; (void)f1;
#elif !defined(DWDP_SCALAR_FMA)
  ffma2(a0, a1, v0, v1, f0, f1);
#else
  a0 = fmaf(v0, f0, a0);
  a1 = fmaf(v1, f1, a1);
#endif
}

// TMEM columns of this thread's lane, N = 16 or 32.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]) {
  if constexpr (N == 16) tmem_ld16(taddr, v);
  else tmem_ld32(taddr, v);
}

// Lane l ends with max over the warp's 32 lanes of v[l] (31 shuffles): at each step a
// lane keeps the half of its array whose index bit matches its own lane bit and
// exchanges the other half with its partner.
__device__ __forceinline__ float warp_transpose_max(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float keep = hi ? v[i + o] : v[i];
      const float send = hi ? v[i] : v[i + o];
      v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return v[0];
}

template <int MODE, int NM, int BNT, int PLANES>
__global__ void __maxnreg__((CfgP<MODE, NM, BNT, PLANES>::MAXREG))
moe_gemm_f8p_kernel(const __grid_constant__ GemmParams p) {
  using C = CfgP<MODE, NM, BNT, PLANES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sW = sB + C::S * C::B_TILE;
  uint8_t* sQ = sW + C::S * C::W_STAGE_BYTES;                                  // [BNT][128] e4m3
  float* sScl = reinterpret_cast<float*>(sQ + C::STAGING);                     // [EPI_WARPS][RING][RSTRIDE]
  float* sRed = sScl + C::EPI_WARPS * C::RING * C::RSTRIDE;                    // [4][BNT]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sRed) + C::RED);
  uint64_t* ld_full = bars;
  uint64_t* ld_empty = ld_full + C::S;
  uint64_t* acc_full = ld_empty + C::S;
  uint64_t* acc_empty = acc_full + C::NSLOT;
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
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], C::EPI_WARPS);
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
      RP_BEGIN
      uint32_t it = 0;
      WorkItem wn = p.items[blockIdx.x];
      for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
        const WorkItem wi = wn;
        if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
        const GroupParams& g = p.g[wi.group];
        const uint8_t* wbase = wi.wtiles;
        const uint32_t b_bytes = (uint32_t)g.box_rows * PLANES * BK8;
        const int nm = min(wi.nmat, C::NMAT);
        for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it) {
          const int s = it % C::S;
          if (!RP_TIMED(0, MBAR_WAIT_P(&ld_empty[s], ((it / C::S) & 1) ^ 1, &s_abort, st, 41 + 8 * MODE))) break;
          mbar_arrive_expect_tx(&ld_full[s], (uint32_t)(nm * kW8TileBytes) + b_bytes);
          for (int m = 0; m < nm; ++m)
            bulk_g2s(sW + s * C::W_STAGE_BYTES + m * kW8TileBytes,
                     wbase + (size_t)m * g.mstride + (size_t)kb * g.kstride, kW8TileBytes, &ld_full[s]);
          tma_load_2d(sB + s * C::B_TILE, &g.tmap_b, kb * BK8, PLANES * wi.row0, &ld_full[s]);
        }
      }
      RP_END(1, 0, 1)
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      RP_BEGIN
      uint32_t it = 0, kc = 0;
      WorkItem wn = p.items[blockIdx.x];
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && !s_abort && ok; item += gridDim.x) {
        const WorkItem wi = wn;
        if (item + (int)gridDim.x < p.cap) wn = p.items[item + gridDim.x];
        const int n_tok = max(16, (wi.nrows + 15) & ~15);
        const uint32_t idesc = idesc_e4m3(BM, PLANES * n_tok);
        const int nm = min(wi.nmat, C::NMAT);
        for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++it, ++kc) {
          const int s = it % C::S;
          const int slot = kc % C::NSLOT;
          if (!RP_TIMED(2, MBAR_WAIT_P(&acc_empty[slot], ((kc / C::NSLOT) & 1) ^ 1, &s_abort, st, 42 + 8 * MODE))) { ok = false; break; }
          if (!RP_TIMED(3, MBAR_WAIT_P(&ld_full[s], (it / C::S) & 1, &s_abort, st, 43 + 8 * MODE))) { ok = false; break; }
          tc_fence_after();
          // a K step of 32 e4m3 (32 bytes) is +2 in the encoded start address
          const uint64_t b_desc0 = smem_desc_sw128(smem_u32(sB + s * C::B_TILE));
          const uint64_t a_desc0 = smem_desc_sw128(smem_u32(sW + s * C::W_STAGE_BYTES));
          const uint32_t d_base = tmem_base + slot * C::SLOT;
          for (int m = 0; m < nm; ++m) {
#pragma unroll
            for (int kk = 0; kk < BK8 / 32; ++kk)
              mma_e4m3_ss(d_base + m * C::NCOL, a_desc0 + (uint64_t)(m * (kW8TileBytes >> 4) + 2 * kk),
                          b_desc0 + (uint64_t)(2 * kk), idesc, kk > 0 ? 1u : 0u);
          }
          mma_commit(&ld_empty[s]);
          mma_commit(&acc_full[slot]);
        }
      }
      RP_END(4, 2, 4)
    }
  } else {
    // ------------------------------------------------------------ epilogue (promotion)
    const int ew = warp - 2;               // 0 .. EPI_WARPS - 1
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int chunk = ew >> 2;
    const int lrow = quad * 32 + lane;     // weight row inside the 128-row block
    const int t0 = chunk * C::TOKW;        // first token of this warp inside the tile
    float* my_scl = sScl + ew * C::RING * C::RSTRIDE;  // this warp's scale ring
    uint32_t kc = 0;
    bool ok = true;
    RP_BEGIN
    for (int item = blockIdx.x; item < n_items && !s_abort && ok; item += gridDim.x) {
      RP_MARK
      const WorkItem wi = p.items[item];  // loaded per item: no registers held across the K loop
      const GroupParams& g = p.g[wi.group];
      const int nm = min(wi.nmat, C::NMAT);
      const int ntk = min(C::TOKW, wi.nrows - t0);  // tokens of this warp (<= 0: none)
      const bool block_w = g.scale_mode == DWDP_SCALE_BLOCK128;
      const int kbn = g.K / 128;                     // K blocks of the projection
      const float* wsc = wi.scales;
      // block-scale index of matrix m at K block kb
      auto wsc_index = [&](int m, int kb) -> int {
        return MODE == 0 ? ((m * (g.R / BM) + wi.rb) * kbn + kb) : ((wi.rb + m) * kbn + kb);
      };
      float acc[C::NMAT][C::TOKW];
#pragma unroll
      for (int m = 0; m < C::NMAT; ++m)
#pragma unroll
        for (int j = 0; j < C::TOKW; ++j) acc[m][j] = 0.f;
      // scale of this lane's token at K block kb (PLANES = 1), prefetched one block ahead
      // K-block kb's scales -> ring slot kb % RING: lane t the scale of token t0 + t (zero past the
      // tile), lanes m < nm the block scale of matrix m (block-scaled weights)
      auto issue = [&](int kb) {
        float* rs = my_scl + (kb % C::RING) * C::RSTRIDE;
        if constexpr (PLANES == 1) {
          const int t = lane < ntk ? lane : 0;
          cp_async4(rs + lane, g.x_scale + (size_t)kb * g.xs_ld + wi.row0 + t0 + t, lane < ntk ? 4u : 0u);
        }
        if (block_w && lane < nm) cp_async4(rs + 32 + lane, wsc + wsc_index(lane, kb), 4u);
        cp_async_commit();
      };
      if (ntk > 0) {
#pragma unroll
        for (int d = 0; d < C::DIST; ++d) {
          if (wi.kb_begin + d < wi.kb_end) issue(wi.kb_begin + d);
          else cp_async_commit();
        }
      }
      // per-row weight scales (CHANNEL / TENSOR), applied after the K loop, loaded now
      const int feat = wi.rb * BM + lrow;
      float s_row[C::NMAT];
#pragma unroll
      for (int m = 0; m < C::NMAT; ++m) {
        s_row[m] = 1.0f;
        if (per_row_scales(g.scale_mode) && m < nm)
          s_row[m] = MODE == 0 ? wsc[m * g.R + feat] : wsc[feat + m * BM];
      }
      for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++kc) {
        const int slot = kc % C::NSLOT;
        const float* rs = my_scl + (kb % C::RING) * C::RSTRIDE;
        float sw_cur[C::NMAT];
#pragma unroll
        for (int m = 0; m < C::NMAT; ++m) sw_cur[m] = 1.0f;
        if (ntk > 0) {
          RP_ADD(10)
          cp_async_wait<C::DIST - 1>();  // this lane's copies of block kb have landed
          __syncwarp();                  // ... and every lane's are visible
#pragma unroll
          for (int m = 0; m < C::NMAT; ++m) sw_cur[m] = (block_w && m < nm) ? rs[32 + m] : 1.0f;
          if constexpr (PLANES == 1) {
            if (block_w) {
              // lane t: the promotion factors of token t0 + t for every matrix
              float* fw = my_scl + (kb % C::RING) * C::RSTRIDE + C::FAC;
              const float sx = rs[lane];
#pragma unroll
              for (int m = 0; m < C::NMAT; ++m) fw[m * 32 + lane] = sx * sw_cur[m];
              __syncwarp();
            }
          }
        }
        __syncwarp();
        RP_ADD(6)
        if (!MBAR_WAIT_P(&acc_full[slot], (kc / C::NSLOT) & 1, &s_abort, st, 44 + 8 * MODE)) { ok = false; break; }
        RP_ADD(5)
        tc_fence_after();
        if (ntk > 0) {
          const uint32_t t_acc = tmem_base + slot * C::SLOT + PLANES * t0 + ((uint32_t)(quad * 32) << 16);
          if constexpr (C::ALL_AT_ONCE) {
            // every matrix's columns in flight at once, one wait
            float v[C::NMAT][C::TCOL];
#pragma unroll
            for (int m = 0; m < C::NMAT; ++m)
#ifdef DWDP_DIAG_NO_TMEM
              for (int j = 0; j < C::TCOL; ++j) v[m][j] = (float)j;
#else
              if (m < nm) tmem_ld<C::TCOL>(t_acc + m * C::NCOL, v[m]);
#endif
            tmem_ld_wait();
            if constexpr (PLANES == 1) {
              // each float4 of token scales serves every matrix
              const float4* f4 = reinterpret_cast<const float4*>(rs);
              if (block_w) {
#pragma unroll
                for (int m = 0; m < C::NMAT; ++m) {
                  if (m < nm) {
                    const float4* fm = reinterpret_cast<const float4*>(rs + C::FAC + m * 32);
#pragma unroll
                    for (int q = 0; q < C::TOKW / 4; ++q) {
                      const float4 f = fm[q];
                      fma_pair(acc[m][4 * q], acc[m][4 * q + 1], v[m][4 * q], v[m][4 * q + 1], f.x, f.y);
                      fma_pair(acc[m][4 * q + 2], acc[m][4 * q + 3], v[m][4 * q + 2], v[m][4 * q + 3], f.z, f.w);
                    }
                  }
                }
              } else {
#pragma unroll
                for (int q = 0; q < C::TOKW / 4; ++q) {
                  const float4 f = f4[q];
#pragma unroll
                  for (int m = 0; m < C::NMAT; ++m) {
                    if (m < nm) {
                      fma_pair(acc[m][4 * q], acc[m][4 * q + 1], v[m][4 * q], v[m][4 * q + 1], f.x, f.y);
                      fma_pair(acc[m][4 * q + 2], acc[m][4 * q + 3], v[m][4 * q + 2], v[m][4 * q + 3], f.z, f.w);
                    }
                  }
                }
              }
            } else {
#pragma unroll
              for (int m = 0; m < C::NMAT; ++m)
                if (m < nm)
#pragma unroll
                  for (int j = 0; j < C::TOKW; ++j)
                    acc[m][j] = fmaf(v[m][2 * j] + v[m][2 * j + 1] * (1.0f / kLoPlaneGain), sw_cur[m], acc[m][j]);
            }
          } else {
            // more columns than registers allow at once: 16 TMEM columns at a time
            constexpr int TPH = 16 / PLANES;  // tokens per 16 columns
#pragma unroll
            for (int m = 0; m < C::NMAT; ++m) {
              if (m < nm) {
#pragma unroll
                for (int hf = 0; hf < C::TCOL / 16; ++hf) {
                  float v[16];
#ifdef DWDP_DIAG_NO_TMEM
                  for (int j = 0; j < 16; ++j) v[j] = (float)j;
#else
                  tmem_ld16(t_acc + m * C::NCOL + 16 * hf, v);
#endif
                  tmem_ld_wait();
                  if constexpr (PLANES == 1) {
                    const float4* f4 =
                        reinterpret_cast<const float4*>(rs + (block_w ? C::FAC + m * 32 : 0) + 16 * hf);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      const float4 f = f4[q];
                      const int j = 16 * hf + 4 * q;
                      fma_pair(acc[m][j], acc[m][j + 1], v[4 * q], v[4 * q + 1], f.x, f.y);
                      fma_pair(acc[m][j + 2], acc[m][j + 3], v[4 * q + 2], v[4 * q + 3], f.z, f.w);
                    }
                  } else {
#pragma unroll
                    for (int j = 0; j < TPH; ++j)
                      acc[m][TPH * hf + j] =
                          fmaf(v[2 * j] + v[2 * j + 1] * (1.0f / kLoPlaneGain), sw_cur[m], acc[m][TPH * hf + j]);
                  }
                }
              }
            }
          }
        }
        RP_ADD(7)
        tc_fence_before();
        __syncwarp();  // every lane is done with ring slot kb % RING and with the TMEM slot
        if (lane == 0) mbar_arrive(&acc_empty[slot]);
        if (ntk > 0) {
          if (kb + C::DIST < wi.kb_end) issue(kb + C::DIST);
          else cp_async_commit();
        }
      }
      if (!ok) break;
      cp_async_wait<0>();

      // ---------------- item epilogue: per-row scales, SwiGLU / routing weight, stores
      RP_ADD(10)
      __syncwarp();
      if constexpr (MODE == 0) {
#ifdef DWDP_DIAG_NO_QOUT
        if constexpr (false) {
#else
        if constexpr (C::QOUT) {
#endif
          // h per the reference executor's bf16 arithmetic, then its (token, 128) amax
          __nv_bfloat162 hp[C::TOKW / 2];  // h of tokens t0 + j, exact in bf16 (the accumulators die here)
#pragma unroll
          for (int j = 0; j < C::TOKW; ++j) {
            const float gb = bf16_round(acc[0][j] * s_row[0]);
            const float ub = bf16_round(acc[1][j] * s_row[1]);
            const float sg = bf16_round(__fdividef(1.0f, 1.0f + __expf(-gb)));
            const float h = j < ntk ? bf16_round(bf16_round(gb * sg) * ub) : 0.f;
            if (j & 1) hp[j >> 1].y = __float2bfloat16_rn(h); else hp[j >> 1].x = __float2bfloat16_rn(h);
          }
          float hq[32];  // |h| of tokens t0 + j (zero past TOKW)
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 f = j < C::TOKW / 2 ? __bfloat1622float2(hp[j]) : make_float2(0.f, 0.f);
            hq[2 * j] = fabsf(f.x);
            hq[2 * j + 1] = fabsf(f.y);
          }
          const float wmax = warp_transpose_max(hq, lane);  // this warp's rows, token t0 + lane
          if (lane < C::TOKW) sRed[quad * BNT + t0 + lane] = wmax;
          named_bar_sync(3, C::EPI_THREADS);
          float tmax = 0.f;
          if (lane < C::TOKW) {
            tmax = sRed[t0 + lane];
#pragma unroll
            for (int q = 1; q < 4; ++q) tmax = fmaxf(tmax, sRed[q * BNT + t0 + lane]);
          }
          const float tsc = __fdiv_rn(fmaxf(tmax, 1e-5f), 448.0f);
          my_scl[lane] = __frcp_rn(tsc);  // quantise by multiplying with the reciprocal
          __syncwarp();
          if (quad == 0 && lane < ntk)
            g.out_scale[(size_t)wi.rb * g.os_ld + wi.row0 + t0 + lane] = tsc;
#pragma unroll
          for (int j = 0; j < C::TOKW; ++j) {
            if (j < ntk) {
              const float hvj = __bfloat162float((j & 1) ? hp[j >> 1].y : hp[j >> 1].x);
              const float q = hvj * my_scl[j];
              sQ[(t0 + j) * BM + lrow] = (uint8_t)__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3);
            }
          }
          named_bar_sync(3, C::EPI_THREADS);
          // e4m3 rows of the tile leave as 16-byte stores
          uint8_t* out8 = reinterpret_cast<uint8_t*>(g.out);
          const int ep = ew * 32 + lane;
          for (int q = ep; q < wi.nrows * (BM / 16); q += C::EPI_THREADS) {
            const int t = q >> 3, ch = q & 7;
            *reinterpret_cast<uint4*>(out8 + (size_t)(wi.row0 + t) * g.R + wi.rb * BM + ch * 16) =
                *reinterpret_cast<const uint4*>(sQ + t * BM + ch * 16);
          }
          named_bar_sync(3, C::EPI_THREADS);  // sQ and sRed are rewritten by the next item
        } else {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out);
#pragma unroll
          for (int j = 0; j < C::TOKW; ++j) {
            if (j < ntk) {
              const float sx = g.x_scale[wi.row0 + t0 + j];
              const float gg = acc[0][j] * (s_row[0] * sx);
              const float uu = acc[1][j] * (s_row[1] * sx);
              out[(size_t)(wi.row0 + t0 + j) * g.R + feat] = __float2bfloat16_rn(silu_fast(gg) * uu);
            }
          }
        }
      } else {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)wi.part * g.part_stride;
#pragma unroll
        for (int j = 0; j < C::TOKW; ++j) {
          if (j < ntk) {
            const int row = wi.row0 + t0 + j;
            float f = g.row_scale != nullptr ? g.row_scale[row] : 1.0f;
            if constexpr (PLANES == 2) f *= g.x_scale[row];
#pragma unroll
            for (int m = 0; m < C::NMAT; ++m)
              if (m < nm) out[(size_t)row * g.R + feat + m * BM] = __float2bfloat16_rn(acc[m][j] * (s_row[m] * f));
          }
        }
      }
      RP_ADD(8)
    }
#ifdef DWDP_PROFILE_ROLES
    if (warp == 2 && lane == 0) RP_END(9, 5, 10)
#endif
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// One e4m3 activation plane scaled per (row, 128 inputs) (DWDP_ACT_BLOCK128, the
// reference's FP8 executor scheme, DWDP/executor/fp8.py:86-115 and
// kernels/fp8_tma.py:99-119) on a CTA pair, for prefill-sized batches.
//
// Same load structure as moe_gemm_f8x2_kernel (two 128-input K blocks per stage: one
// 3-D TMA box of activation rows and one bulk copy of weight tiles per CTA, 32 KB per
// K block per SM), but A holds 128 distinct tokens per CTA (items of up to 256
// tokens), so one MMA column carries one token instead of a hi/lo pair: half the MMA
// work of the hi/lo mode per token. The activation scale changes every 128 inputs,
// so every K block is multiplied into its own TMEM slot (two slots of 256 columns,
// the tensor core one block ahead of the epilogue) and the epilogue warps fold it
// into fp32 registers:  acc += slot * (s_x[token][kb] * s_w[kb])  (s_w only for
// 128x128 block-scaled weights; per-row weight scales are applied once at the end).
// Epilogue warp (quadrant q = warp % 4, half hw): TMEM lanes 32q..32q+31 = tokens, and
//   MODE 0: gate and up features [64 hw, 64 hw + 64) of the item's 128-feature block
//           (TMEM columns 64 hw.. and 128 + 64 hw..). At the end: SwiGLU in the
//           reference executor's bf16 arithmetic and re-quantisation per (token, 128
//           features) into the down projection's e4m3 rows + scales; the two halves of a
//           quadrant exchange their |h| maxima through shared memory behind a bounded
//           flag wait (no CTA-wide barrier an aborting warp could leave waiting);
//   MODE 1: output columns [128 hw, 128 hw + 128) = down row block rb + hw, times the
//           routing weight, bf16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}

// logistic function from the hardware tanh: 1 / (1 + e^-x) = 0.5 + 0.5 tanh(x / 2), one MUFU
// operation instead of an exponential and a reciprocal (max abs error ~2^-11, below bf16's step)
__device__ __forceinline__ float sigmoid_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return fmaf(0.5f, t, 0.5f);
}

struct CfgX2P {
  static constexpr int KPS = 2;                       // K blocks per stage
  static constexpr int A_TILE = 128 * BK8;            // 128 tokens x 128 inputs
  static constexpr int B_TILE = kW8TileBytes;         // 128 weight rows x 128 inputs
  static constexpr int STAGE_A = KPS * A_TILE;
  static constexpr int STAGE_B = KPS * B_TILE;
  static constexpr int STAGE = STAGE_A + STAGE_B;
  static constexpr int S = 3;
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int THREADS = (2 + EPI_WARPS) * 32;
  static constexpr int SLOT_COLS = 256;               // one K block's 256 x 256 product per CTA pair
  static constexpr int NSLOT = 2;
  static constexpr int RED_BYTES = 2 * 2 * 128 * 4 + 2 * 2 * 4 * 4;  // |h| maxima + flags
  // per-warp ring of K-block scales filled DIST blocks ahead by asynchronous copies:
  // a slot holds [32 token scales | 2 weight-block scales | pad]
  static constexpr int RING = 4, DIST = 3, RSTRIDE = 36;
  static constexpr int SCL_BYTES = EPI_WARPS * RING * RSTRIDE * 4;
  // per-warp copy of the item's per-row weight scales (its 128 accumulator columns)
  static constexpr int ROW_BYTES = EPI_WARPS * 128 * 4;
  static constexpr int SMEM_BYTES = S * STAGE + RED_BYTES + SCL_BYTES + ROW_BYTES + 1024 + 512;
  static constexpr uint32_t kFlagPolls = 1u << 24;    // bound of the halves' exchange wait (polls)
  // TMEM columns per load: 16 keeps the 128 accumulators + the loaded columns inside the
  // 168 registers a thread of a 10-warp CTA gets (3 warps share the fullest sub-partition)
#ifdef DWDP_X2P_CHUNK
  static constexpr int CHUNK = DWDP_X2P_CHUNK;
#else
  static constexpr int CHUNK = 16;
#endif
};

#ifdef DWDP_PROFILE_ROLES
// Diagnostic build only: cycles per activity of moe_gemm_f8x2p_kernel's roles in
// g_role_cycles[cta][32 * MODE + slot] (producer 0-1, leader / relay 2-5, epilogue warp 2: 6-10).
#define XP_DECL unsigned long long xp_[12] = {}; long long xpt_ = clock64();
#define XP_ACC(slot) { const long long n_ = clock64(); xp_[slot] += (unsigned long long)(n_ - xpt_); xpt_ = n_; }
#define XP_STORE(lo, hi) { for (int q_ = lo; q_ <= hi; ++q_) g_role_cycles[blockIdx.x][32 * MODE + q_] = xp_[q_]; }
#else
#define XP_DECL
#define XP_ACC(slot)
#define XP_STORE(lo, hi)
#endif

template <int MODE>
__global__ void __launch_bounds__(CfgX2P::THREADS, 1) moe_gemm_f8x2p_kernel(const __grid_constant__ GemmParams p) {
  using C = CfgX2P;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::S * C::STAGE_A;
  float* sRed = reinterpret_cast<float*>(smem + C::S * C::STAGE);                  // [2 buf][2 half][128 tok]
  volatile int* sFlag = reinterpret_cast<volatile int*>(sRed + 2 * 2 * 128);       // [2 buf][2 half][4 quad]
  float* sScl = reinterpret_cast<float*>(smem + C::S * C::STAGE + C::RED_BYTES);   // [EPI_WARPS][RING][RSTRIDE]
  float* sRow = sScl + C::EPI_WARPS * C::RING * C::RSTRIDE;                         // [EPI_WARPS][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::S * C::STAGE + C::RED_BYTES + C::SCL_BYTES + C::ROW_BYTES);
  uint64_t* full = bars;                       // local loads of stage s landed
  uint64_t* empty = full + C::S;               // the pair's MMAs read stage s (leader commit, both CTAs)
  uint64_t* peer_full = empty + C::S;          // leader only: the peer's stage s landed
  uint64_t* acc_full = peer_full + C::S;       // TMEM slot holds a K block's product (leader commit, both)
  uint64_t* acc_empty = acc_full + C::NSLOT;   // this CTA's epilogue read the slot
  uint64_t* peer_acc_empty = acc_empty + C::NSLOT;  // leader only: the peer's epilogue read the slot
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_rank();
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  DeviceStatus* st = p.st;
  griddep_launch();
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < C::S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&peer_full[i], 1);
    }
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], C::EPI_WARPS);  // one arrival per epilogue warp
      mbar_init(&peer_acc_empty[i], 1);
    }
    fence_barrier_init();
  }
  if (threadIdx.x < 16) sFlag[threadIdx.x] = 0;
  if (warp == 1) {
    tmem_alloc2(&s_tmem_base, C::NSLOT * C::SLOT_COLS);
    tmem_relinquish2();
  }
  if (warp == 0 && lane == 0) {
    if (p.g[0].enabled) prefetch_tmap(&p.g[0].tmap_b);
    if (p.g[1].enabled) prefetch_tmap(&p.g[1].tmap_b);
  }
  tc_fence_before();
  cluster_sync_all();  // barriers and flags of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = s_tmem_base;
  griddep_wait();
  const int n_items = *p.n_items;
  if (warp == 0) {
    // ------------------------------------------------------------ producer (each CTA its halves)
    if (lane == 0) {
      XP_DECL
      uint32_t it = 0;
      for (int item = cid; item < n_items && !s_abort; item += ncl) {
        const WorkItem wi = p.items[item];
        const GroupParams& g = p.g[wi.group];
        const int h = min(128, (wi.nrows + 1) >> 1);  // tokens of CTA 0; CTA 1 takes the rest
        const int tok0 = wi.row0 + (int)rank * h;
        const uint8_t* wsrc = wi.wtiles + (size_t)rank * g.mstride;
        for (int kb = wi.kb_begin; kb < wi.kb_end; kb += C::KPS, ++it) {
          const int s = it % C::S;
          const int nkb = min(C::KPS, wi.kb_end - kb);
          XP_ACC(1)
          if (!mbar_wait(&empty[s], ((it / C::S) & 1) ^ 1, &s_abort, st, 121 + 8 * MODE)) break;
          XP_ACC(0)
          // the activation box always lands whole (K blocks past the end read as zeros)
          mbar_arrive_expect_tx(&full[s], (uint32_t)(C::STAGE_A + nkb * C::B_TILE));
          if (g.kstride == C::B_TILE) {
            bulk_g2s(sB + s * C::STAGE_B, wsrc + (size_t)kb * g.kstride, nkb * C::B_TILE, &full[s]);
          } else {
            for (int q = 0; q < nkb; ++q)
              bulk_g2s(sB + s * C::STAGE_B + q * C::B_TILE, wsrc + (size_t)(kb + q) * g.kstride, C::B_TILE, &full[s]);
          }
          tma_load_3d(sA + s * C::STAGE_A, &g.tmap_b, 0, tok0, kb, &full[s]);
        }
      }
      XP_ACC(1)
      XP_STORE(0, 1)
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------------ MMA issuer (leader)
      XP_DECL
      uint32_t it = 0, kc = 0;
      const uint32_t idesc = idesc_e4m3(256, 256);
      bool ok = true;
      for (int item = cid; item < n_items && !s_abort && ok; item += ncl) {
        const WorkItem wi = p.items[item];
        for (int kb = wi.kb_begin; kb < wi.kb_end && ok; kb += C::KPS, ++it) {
          const int s = it % C::S;
          const int nkb = min(C::KPS, wi.kb_end - kb);
          const uint32_t fp = (it / C::S) & 1;
          XP_ACC(5)
          if (!mbar_wait(&full[s], fp, &s_abort, st, 122 + 8 * MODE) ||
              !mbar_wait(&peer_full[s], fp, &s_abort, st, 123 + 8 * MODE)) {
            ok = false;
            break;
          }
          XP_ACC(2)
          for (int q = 0; q < nkb; ++q, ++kc) {
            const int slot = kc & 1;
            const uint32_t par = ((kc >> 1) & 1) ^ 1;
            XP_ACC(5)
            if (!mbar_wait(&acc_empty[slot], par, &s_abort, st, 124 + 8 * MODE)) {
              ok = false;
              break;
            }
            XP_ACC(3)
            if (!mbar_wait(&peer_acc_empty[slot], par, &s_abort, st, 125 + 8 * MODE)) {
              ok = false;
              break;
            }
            XP_ACC(4)
            tc_fence_after();
            const uint32_t d = tmem_base + slot * C::SLOT_COLS;
            const uint64_t ad = smem_desc_sw128(smem_u32(sA + s * C::STAGE_A + q * C::A_TILE));
            const uint64_t bd = smem_desc_sw128(smem_u32(sB + s * C::STAGE_B + q * C::B_TILE));
#pragma unroll
            for (int kk = 0; kk < BK8 / 32; ++kk)
              mma2_e4m3_ss(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), idesc, kk > 0 ? 1u : 0u);
            mma2_commit_mc(&acc_full[slot], 0x3);
          }
          if (ok) mma2_commit_mc(&empty[s], 0x3);
        }
      }
      XP_ACC(5)
      XP_STORE(2, 5)
    } else if (lane == 0) {
      // ------------------------------------------------------------ relay (peer): local phases -> leader
      XP_DECL
      uint32_t it = 0, kc = 0;
      bool ok = true;
      for (int item = cid; item < n_items && !s_abort && ok; item += ncl) {
        const WorkItem wi = p.items[item];
        for (int kb = wi.kb_begin; kb < wi.kb_end && ok; kb += C::KPS, ++it) {
          const int s = it % C::S;
          const int nkb = min(C::KPS, wi.kb_end - kb);
          XP_ACC(5)
          if (!mbar_wait(&full[s], (it / C::S) & 1, &s_abort, st, 126 + 8 * MODE)) {
            ok = false;
            break;
          }
          XP_ACC(2)
          mbar_arrive_remote(&peer_full[s], 0);
          for (int q = 0; q < nkb; ++q, ++kc) {
            if (kc < 2) continue;  // both slots start free
            const int slot = kc & 1;
            XP_ACC(5)
            if (!mbar_wait(&acc_empty[slot], ((kc >> 1) & 1) ^ 1, &s_abort, st, 127 + 8 * MODE)) {
              ok = false;
              break;
            }
            XP_ACC(3)
            mbar_arrive_remote(&peer_acc_empty[slot], 0);
          }
        }
      }
      XP_ACC(5)
      XP_STORE(2, 5)
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;                 // TMEM lanes 32 quad .. 32 quad + 31
    const int hw = (warp - 2) >> 2;            // column half of the item this warp folds
    const int t_cta = quad * 32 + lane;        // token of this lane inside the CTA's 128
    uint32_t kc = 0;
    int li = 0;
    XP_DECL
    for (int item = cid; item < n_items; item += ncl, ++li) {
      if (__any_sync(0xffffffffu, s_abort != 0)) break;  // warp-uniform exit
      const WorkItem wi = p.items[item];
      const GroupParams& g = p.g[wi.group];
      const int h = min(128, (wi.nrows + 1) >> 1);
      const int n_my = rank == 0 ? h : wi.nrows - h;
      const bool live = t_cta < n_my;
      const int tok = wi.row0 + (int)rank * h + t_cta;
      const bool block_w = g.scale_mode == DWDP_SCALE_BLOCK128;
      const int kbn = g.K / 128;
      // K block kb's scales -> ring slot kb % RING: lane t the scale of its token (zero past the
      // tile), lanes m < 2 the weight-block scale of matrix m (MODE 0: gate, up; MODE 1: block
      // rb + hw in both) when the weights are block-scaled
      float* ring = sScl + (warp - 2) * C::RING * C::RSTRIDE;
      auto issue = [&](int kb) {
        float* rs = ring + (kb % C::RING) * C::RSTRIDE;
        cp_async4(rs + lane, g.x_scale + (size_t)kb * g.xs_ld + (live ? tok : wi.row0), live ? 4u : 0u);
        if (block_w && lane < 2) {
          const int blk = MODE == 0 ? (lane * (g.R / BM) + wi.rb) : (wi.rb + hw);
          cp_async4(rs + 32 + lane, wi.scales + (size_t)blk * kbn + kb, 4u);
        }
        cp_async_commit();
      };
      // per-row weight scales of this warp's columns, in the first group: one 16-byte copy per lane
      // (MODE 0: lanes 0-15 gate, 16-31 up of features fb..fb+63; MODE 1: features fb..fb+127)
      const bool per_row = per_row_scales(g.scale_mode);
      const int fb = MODE == 0 ? wi.rb * BM + 64 * hw : wi.rb * BM + 128 * hw;
      float* row_s = sRow + (warp - 2) * 128;
      if (per_row) {
        const float* src = MODE == 0 ? wi.scales + (lane < 16 ? fb + 4 * lane : g.R + fb + 4 * (lane - 16))
                                     : wi.scales + fb + 4 * lane;
        cp_async16(row_s + 4 * lane, src);
      }
#pragma unroll
      for (int d = 0; d < C::DIST; ++d) {
        if (wi.kb_begin + d < wi.kb_end) issue(wi.kb_begin + d);
        else cp_async_commit();
      }
      float acc[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.f;
      bool ok = true;
      XP_ACC(10)
      for (int kb = wi.kb_begin; kb < wi.kb_end; ++kb, ++kc) {
        const int slot = kc & 1;
        // one lane per warp polls the barrier (256 pollers per K block would crowd shared memory)
        int got = 1;
        XP_ACC(6)
        if (lane == 0) got = mbar_wait(&acc_full[slot], (kc >> 1) & 1, &s_abort, st, 128 + 8 * MODE) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          break;
        }
        XP_ACC(7)
        // the block's scales (their copies overlapped the wait above)
        cp_async_wait<C::DIST - 1>();  // this lane's copies of block kb have landed
        __syncwarp();                  // ... and every lane's are visible
        const float* rs = ring + (kb % C::RING) * C::RSTRIDE;
        const float sx = rs[lane];
        const float f0 = block_w ? sx * rs[32] : sx;
        const float f1 = block_w ? sx * rs[33] : sx;
        tc_fence_after();
        const uint32_t t_slot = tmem_base + slot * C::SLOT_COLS + ((uint32_t)(quad * 32) << 16);
#pragma unroll
        for (int c = 0; c < 128 / CfgX2P::CHUNK; ++c) {
          constexpr int CH = CfgX2P::CHUNK;
          const int a0 = CH * c;  // first accumulator of the chunk
          const int col = MODE == 0 ? ((a0 >> 6) * 128 + 64 * hw + (a0 & 63)) : (128 * hw + a0);
          const float f = (MODE == 0 && a0 >= 64) ? f1 : f0;
          float v[CH];
          tmem_ld<CH>(t_slot + col, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < CH; j += 2) fma_pair(acc[a0 + j], acc[a0 + j + 1], v[j], v[j + 1], f, f);
        }
        tc_fence_before();
        __syncwarp();  // every lane is done with the TMEM slot and with ring slot kb % RING
        if (lane == 0) mbar_arrive(&acc_empty[slot]);
        XP_ACC(8)
        if (kb + C::DIST < wi.kb_end) issue(kb + C::DIST);
        else cp_async_commit();
      }
      cp_async_wait<0>();
      __syncwarp();  // every lane's copies (ring, per-row scales) are visible
      XP_ACC(6)
      if (!ok) break;
      if constexpr (MODE == 0) {
        // h per the reference executor's bf16 arithmetic; acc[j] = gate, acc[64 + j] = up of
        // feature fb + j
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
          float4 sg = make_float4(1.f, 1.f, 1.f, 1.f), su = sg;
          if (per_row) {
            sg = *reinterpret_cast<const float4*>(row_s + j);
            su = *reinterpret_cast<const float4*>(row_s + 64 + j);
          }
          const float gs[4] = {sg.x, sg.y, sg.z, sg.w}, us[4] = {su.x, su.y, su.z, su.w};
          // pairs of features in bf16x2: a product of two bf16 values is exact in fp32, so the
          // packed bf16 multiply rounds exactly as bf16(fp32 product) does
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const __nv_bfloat162 g2 = __floats2bfloat162_rn(acc[j + e] * gs[e], acc[j + e + 1] * gs[e + 1]);
            const __nv_bfloat162 u2 =
                __floats2bfloat162_rn(acc[64 + j + e] * us[e], acc[64 + j + e + 1] * us[e + 1]);
            const float2 gf = __bfloat1622float2(g2);
            const __nv_bfloat162 s2 = __floats2bfloat162_rn(sigmoid_tanh(gf.x), sigmoid_tanh(gf.y));
            const float2 hf = __bfloat1622float2(__hmul2(__hmul2(g2, s2), u2));
            acc[j + e] = hf.x;  // h replaces the gate accumulators
            acc[j + e + 1] = hf.y;
            amax = fmaxf(amax, fmaxf(fabsf(hf.x), fabsf(hf.y)));
          }
        }
        // (token, 128-feature) amax: exchange with the other half of this quadrant
        const int b = li & 1;
        sRed[(b * 2 + hw) * 128 + t_cta] = live ? amax : 0.f;
        __syncwarp();
        __threadfence_block();
        if (lane == 0) sFlag[(b * 2 + hw) * 4 + quad] = li + 1;
        int seen = 1;
        if (lane == 0) {
          uint32_t n = 0;
          while (sFlag[(b * 2 + (hw ^ 1)) * 4 + quad] != li + 1) {
            if (++n >= C::kFlagPolls || s_abort) {
              seen = 0;
              break;
            }
          }
        }
        seen = __shfl_sync(0xffffffffu, seen, 0);
        if (!seen) {
          if (lane == 0 && !s_abort) {
            s_abort = 1;
            record_error(st, DWDP_ERR_DEVICE_TIMEOUT, 129 + 8 * MODE, li);
          }
          break;
        }
        __threadfence_block();
        const float tmax = fmaxf(amax, sRed[(b * 2 + (hw ^ 1)) * 128 + t_cta]);
        const float tsc = __fdiv_rn(fmaxf(tmax, 1e-5f), 448.0f);
        const float rcp = __frcp_rn(tsc);  // quantise by multiplying with the reciprocal
        if (live) {
          if (hw == 0) g.out_scale[(size_t)wi.rb * g.os_ld + tok] = tsc;
          uint8_t* dst = reinterpret_cast<uint8_t*>(g.out) + (size_t)tok * g.R + fb;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 16 * q + 4 * e;
              const uint32_t lo = (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(acc[j] * rcp, acc[j + 1] * rcp),
                                                                      __NV_SATFINITE, __NV_E4M3);
              const uint32_t hi = (uint32_t)__nv_cvt_float2_to_fp8x2(
                  make_float2(acc[j + 2] * rcp, acc[j + 3] * rcp), __NV_SATFINITE, __NV_E4M3);
              w[e] = lo | (hi << 16);
            }
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else {
        if (live) {
          const float rw = g.row_scale != nullptr ? g.row_scale[tok] : 1.0f;
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)wi.part * g.part_stride +
                               (size_t)tok * g.R + fb;
#pragma unroll
          for (int j = 0; j < 128; j += 8) {
            float4 s0 = make_float4(1.f, 1.f, 1.f, 1.f), s1 = s0;
            if (per_row) {
              s0 = *reinterpret_cast<const float4*>(row_s + j);
              s1 = *reinterpret_cast<const float4*>(row_s + j + 4);
            }
            const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 yv = __floats2bfloat162_rn(acc[j + 2 * e] * (sc[2 * e] * rw),
                                                              acc[j + 2 * e + 1] * (sc[2 * e + 1] * rw));
              w[e] = *reinterpret_cast<const uint32_t*>(&yv);
            }
            reinterpret_cast<uint4*>(out)[j / 8] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      XP_ACC(9)
    }
    if (warp == 2 && lane == 0) { XP_STORE(6, 10) }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // both CTAs done: the leader's MMAs and both epilogues
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, C::NSLOT * C::SLOT_COLS);
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
  int scale_rowmajor;        // single-plane quantiser: scales [rows][K / 128] instead of [K / 128][rows]
};
struct QuantParams {
  QuantSeg seg[2];
  DeviceStatus* st;
  int per_warp;  // 1: one warp per row (many rows); 0: one CTA per row (few, long rows)
  int blk;       // 1: one e4m3 plane, scales per (row, 128): dst [rows, K], scale [K / 128][rows]
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

// One e4m3 plane with one scale per (row, 128 channels), as
// DWDP/executor/fp8.py:86-115 quantize_activations_blockwise computes it:
// scale = max(amax of the block, 1e-5) / 448 and q = e4m3(v / scale), both with
// IEEE division and round-to-nearest-even, so the bytes and scales equal the
// reference's. One warp handles 512 columns of one row (a lane 16 consecutive
// elements, 8 lanes per 128-block); scales are stored transposed, [K / 128][rows],
// so that the GEMM epilogue reads one K block's scales of consecutive rows.
__device__ __forceinline__ void quant_seg_blk(const QuantSeg& g, int row, int part, DeviceStatus* st) {
  const int lane = threadIdx.x & 31;
  int64_t sr = row;
  if (g.row_index != nullptr) {
    sr = g.row_index[row];
    if (sr < 0 || sr >= g.src_rows) {
      if (lane == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 213, row);
      sr = -1;
    }
  }
  const int c = part * 512 + lane * 16;
  const bool in = c < g.K;
  uint4 a = make_uint4(0, 0, 0, 0), b = make_uint4(0, 0, 0, 0);
  if (in && sr >= 0) {
    const __nv_bfloat16* src = g.src + (size_t)sr * g.K + c;
    a = *reinterpret_cast<const uint4*>(src);
    b = *reinterpret_cast<const uint4*>(src + 8);
  }
  float amax = amax8(b, amax8(a, 0.f));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  const float scale = __fdiv_rn(fmaxf(amax, 1e-5f), 448.0f);
  if (!in) return;
  const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
  auto q2 = [&](const __nv_bfloat162 v) -> uint32_t {
    const float2 f = __bfloat1622float2(v);
    const float2 qv = make_float2(__fdiv_rn(f.x, scale), __fdiv_rn(f.y, scale));
    return (uint32_t)__nv_cvt_float2_to_fp8x2(qv, __NV_SATFINITE, __NV_E4M3);
  };
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 lo = k < 2 ? pa[2 * k] : pb[2 * k - 4];
    const __nv_bfloat162 hi = k < 2 ? pa[2 * k + 1] : pb[2 * k - 3];
    w[k] = q2(lo) | (q2(hi) << 16);
  }
  *reinterpret_cast<uint4*>(g.dst + (size_t)row * g.K + c) = make_uint4(w[0], w[1], w[2], w[3]);
  if ((lane & 7) == 0) {
    const size_t si = g.scale_rowmajor ? (size_t)row * (g.K >> 7) + (c >> 7) : (size_t)(c >> 7) * g.rows + row;
    g.scale[si] = scale;
  }
}

__device__ __forceinline__ void quant_rows_blk(const QuantParams& q, int block, int nblocks) {
  constexpr int kW = kPlanThreads / 32;
  const int np0 = (q.seg[0].K + 511) / 512, np1 = (q.seg[1].K + 511) / 512;
  const int u0 = q.seg[0].rows * np0;
  const int total = u0 + q.seg[1].rows * np1;
  for (int u = block * kW + (int)(threadIdx.x >> 5); u < total; u += nblocks * kW) {
    if (u < u0) quant_seg_blk(q.seg[0], u / np0, u % np0, q.st);
    else quant_seg_blk(q.seg[1], (u - u0) / np1, (u - u0) % np1, q.st);
  }
}

// Rows of both segments, one per `first + i * stride` unit (a warp or a CTA).
__device__ __forceinline__ void quant_rows(const QuantParams& q, int block, int nblocks) {
  if (q.blk) {
    quant_rows_blk(q, block, nblocks);
    return;
  }
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

// 2-D map over e4m3 activation rows: `planes` = 2 for the interleaved hi/lo planes
// [2 * rows, cols] (box {128, 2 * box_rows}), 1 for one plane [rows, cols].
// The same planes as a 3-D map {128 inputs, plane rows, K blocks}: one box brings two
// consecutive 128-input tiles of box_rows tokens (two 16 KB tiles back to back in shared
// memory), for the CTA-pair kernels with two K blocks per stage.
bool make_tmap_planes3(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int planes) {
  auto enc = get_encode_fn();
  if (enc == nullptr || rows <= 0 || cols % BK8) return false;
  cuuint64_t dims[3] = {(cuuint64_t)BK8, (cuuint64_t)(planes * rows), (cuuint64_t)(cols / BK8)};
  cuuint64_t strides[2] = {(cuuint64_t)cols, (cuuint64_t)BK8};
  cuuint32_t box[3] = {(cuuint32_t)BK8, (cuuint32_t)(planes * box_rows), 2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_planes(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int planes) {
  auto enc = get_encode_fn();
  if (enc == nullptr || rows <= 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)(planes * rows)};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)BK8, (cuuint32_t)(planes * box_rows)};
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
  // activation scales: one per row (hi/lo) or per (row, 128 inputs) (BLOCK128)
  w.sx_r = o; o = align256(o + (size_t)N * (H / 128) * 4);
  w.sx_s = o; o = align256(o + (size_t)T * (H / 128) * 4);
  w.sh_r = o; o = align256(o + (size_t)N * (I / 128) * 4);
  w.sh_s = o; o = align256(o + (size_t)T * (Isz / 128) * 4);
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

// CTA-pair kernels: clusters of two consecutive CTAs (grid must be even), programmatic launch.
template <typename Kfn>
int launch_pair(Kfn kfn, int threads, int smem_bytes, const GemmParams& prm, int grid, cudaStream_t stream) {
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
    return DWDP_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid & ~1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = 2;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kfn, prm) == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

template <int MODE, int KPS>
int launch_gemm_f8x2(const GemmParams& prm, int grid, cudaStream_t stream) {
  using C = CfgX2<MODE, KPS>;
  return launch_pair(moe_gemm_f8x2_kernel<MODE, KPS>, C::THREADS, C::SMEM_BYTES, prm, grid, stream);
}

template <int MODE>
int launch_gemm_f8x2p(const GemmParams& prm, int grid, cudaStream_t stream) {
  return launch_pair(moe_gemm_f8x2p_kernel<MODE>, CfgX2P::THREADS, CfgX2P::SMEM_BYTES, prm, grid, stream);
}

// One warp per row once the rows fill every SM's warps; below that a CTA per
// row (decode: a few long rows want more loads in flight than one warp has).
constexpr int64_t kQuantWarpRows = 148 * 8;
inline int quant_per_warp(int64_t rows) { return rows >= kQuantWarpRows ? 1 : 0; }
inline int quant_blocks(int64_t rows) {
  const int64_t b = quant_per_warp(rows) ? (rows + kPlanThreads / 32 - 1) / (kPlanThreads / 32) : rows;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16));
}

// one warp per (row, 512-column part) for the single-plane quantiser
inline int quant_blocks_blk(int64_t units) {
  const int64_t b = (units + kPlanThreads / 32 - 1) / (kPlanThreads / 32);
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16));
}

template <int MODE>
int launch_gemm(const GemmParams& prm, int grid, cudaStream_t stream) {
  using C = Cfg<MODE>;
  auto kfn = moe_gemm_kernel<MODE>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return DWDP_ERR_CUDA;
  return launch_chained(kfn, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, stream, 1u, prm) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

template <int MODE, int NM, int BNT, int PLANES>
int launch_gemm_f8p(const GemmParams& prm, int grid, cudaStream_t stream) {
  using C = CfgP<MODE, NM, BNT, PLANES>;
  auto kfn = moe_gemm_f8p_kernel<MODE, NM, BNT, PLANES>;
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
  // Kernel family: per-row-scaled e4m3 weights with hi/lo activations need no promotion
  // (moe_gemm_f8_kernel); activations scaled per (row, 128) or block-scaled weights promote
  // every 128-wide K block (moe_gemm_f8p_kernel, one or two activation planes); bf16
  // weights run kind::f16 MMAs (moe_gemm_kernel).
  const bool act_blk = fp8 && routed->act_quant == DWDP_ACT_BLOCK128;
  const bool hilo_native = fp8 && !act_blk && per_row_scales(routed->scale_mode);
  const bool promote = fp8 && !hilo_native;
  const int planes = act_blk ? 1 : 2;  // e4m3 activation planes (fp8 paths)
  const int bk = fp8 ? BK8 : BK;
  const int64_t N = shared_only ? 0 : T * K;  // routed rows
  // Token tiles: 64. 128-token tiles halve the weight traffic per FLOP, but measured slower:
  // hi/lo keeps one TMEM accumulator buffer for gate/up and a 3-deep ring; one plane needs
  // sixteen promotion warps whose 96-register budget spills the accumulators.
  // DWDP_WIDE_TILES=1 selects them for tuning.
  bool wide = false;
  if (const char* v = getenv("DWDP_WIDE_TILES"))  // tuning override
    wide = (hilo_native || act_blk) && v[0] == '1';
  const int bn = fp8 ? (wide ? 128 : BN8) : BN_MAX;
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
  // e4m3 64-token tiles at prefill sizes: a down item covers two consecutive 128-row blocks
  // (one activation tile for two MMAs, half the activation traffic per FLOP). Decode keeps
  // single blocks: there the halved item count would leave SMs idle or unevenly loaded (pairs
  // need ~4 waves of items). 128-token tiles always run single down blocks.
  const int sms_now = dwdp_device_sm_count();
  const int64_t est_tiles = N / BN8 + std::min<int64_t>(E, N) + (has_shared ? (T + BN8 - 1) / BN8 * parts : 0);
  bool pair_dn = fp8 && !(act_blk && wide) && est_tiles * ((H / BM + 1) / 2) >= 4LL * std::max(1, sms_now);
  if (const char* v = getenv("DWDP_PAIR_DOWN"))  // tuning override
    pair_dn = fp8 && !(act_blk && wide) && v[0] == '1';
  // Prefill-sized hi/lo batches run on CTA pairs (moe_gemm_f8x2_kernel: 128-token tiles, 64 per
  // CTA, down items always two 128-row blocks). DWDP_PAIR_CTA=0|1 overrides the default.
  bool use_pair = false, use_pair_blk = false;
  {
    static const int pair_env = [] {
      const char* v = getenv("DWDP_PAIR_CTA");
      return v != nullptr ? atoi(v) : 1;
    }();
    // tuning: routed rows from which the pairs run (read every call, so tests can move it)
    const char* pmin = getenv("DWDP_PAIR_MIN_ROWS");
    const long long pair_min = pmin != nullptr ? atoll(pmin) : 148LL * 64;
    use_pair = pair_env == 1 && hilo_native && !wide && (H / BM) % 2 == 0 && N >= pair_min;
    // the reference's single-plane scheme on CTA pairs (moe_gemm_f8x2p_kernel: 256-token
    // tiles, 128 per CTA, per-K-block promotion); DWDP_PAIR_BLK=0 keeps the one-CTA kernels
    static const int pair_blk_env = [] {
      const char* v = getenv("DWDP_PAIR_BLK");
      return v != nullptr ? atoi(v) : 1;
    }();
    use_pair_blk = pair_env == 1 && pair_blk_env == 1 && act_blk && !wide && (H / BM) % 2 == 0 && N >= pair_min;
  }
  static const int pair_kps = [] {  // tuning: K blocks per stage of the pair kernels (1 or 2)
    const char* v = getenv("DWDP_PAIR_KPS");
    return v != nullptr && atoi(v) == 1 ? 1 : 2;
  }();
  if (use_pair || use_pair_blk) pair_dn = true;
  const int dn_items_per_tile = pair_dn ? (H / BM + 1) / 2 : H / BM;
  pp.rb_gu_r = I / BM; pp.rb_dn_r = dn_items_per_tile;
  pp.rb_gu_s = has_shared ? Is / BM : 0; pp.rb_dn_s = has_shared ? dn_items_per_tile : 0;
  pp.dn_pair = pair_dn ? 1 : 0; pp.blocks_dn = H / BM;
  pp.kb_gu = H / bk; pp.kb_dn_r = I / bk; pp.kb_dn_s = has_shared ? Is / bk : 0;
  pp.sdn_parts = has_shared ? parts : 0;
  pp.bn_max = use_pair ? 128 : use_pair_blk ? 256 : bn;
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
  const int64_t q_rows = N + (has_shared ? T : 0);
  qx.per_warp = qh.per_warp = quant_per_warp(q_rows);
  qx.blk = act_blk ? 1 : 0;
  const bool indexed = packed_hidden == nullptr;
  if (indexed && packed_tok == nullptr && N > 0) return DWDP_ERR_INVALID_ARGUMENT;
  if (fp8) {
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
  int qx_blocks = 0;
  if (fp8) qx_blocks = act_blk ? quant_blocks_blk(N * ((H + 511) / 512) + (has_shared ? T * ((H + 511) / 512) : 0))
                               : quant_blocks(q_rows);
  if (launch_chained(prep_kernel, dim3(kPlanBlocks + qx_blocks), dim3(kPlanThreads), 0, stream, 1u, pp, qx) !=
      cudaSuccess)
    return DWDP_ERR_CUDA;

  // The activation box must cover the largest tile: a routed tile holds at most
  // min(T * K, bn) rows (an expert may be picked more than once per token), a
  // shared tile at most min(T, bn).
  const int box_r = use_pair ? 64 : use_pair_blk ? 128 : box_rows_for(N, bn);
  const int box_s = use_pair ? 64 : use_pair_blk ? 128 : box_rows_for(T, bn);
  auto map = [&](CUtensorMap* m, const void* bf16, size_t planes_off, int64_t rows, int64_t cols, int box) {
    if (fp8 && ((use_pair && pair_kps == 2) || use_pair_blk))
      return make_tmap_planes3(m, ws + planes_off, rows, cols, box, planes);
    return fp8 ? make_tmap_planes(m, ws + planes_off, rows, cols, box, planes) : make_tmap(m, bf16, rows, cols, box);
  };
  GemmParams gu{}, dn{};
  gu.g[0].enabled = N > 0;
  if (N > 0 && !map(&gu.g[0].tmap_b, packed_hidden, L.x8_r, N, H, box_r)) return DWDP_ERR_CUDA;
  gu.g[0].w = routed->w13; gu.g[0].s = routed->s13; gu.g[0].row_scale = nullptr;
  gu.g[0].out = act_blk ? static_cast<void*>(ws + L.h8_r) : static_cast<void*>(h_r);
  gu.g[0].out_scale = sh_r; gu.g[0].os_ld = N;
  gu.g[0].x_scale = sx_r; gu.g[0].xs_ld = N;
  gu.g[0].K = H; gu.g[0].R = I; gu.g[0].scale_mode = routed->scale_mode; gu.g[0].box_rows = box_r;
  // e4m3 tiles: a row block's gate tiles along K, then its up tiles; down row blocks are K/128 tiles apart
  gu.g[0].mstride = (long long)(H / BK8) * kW8TileBytes; gu.g[0].kstride = kW8TileBytes;
  gu.g[1].enabled = has_shared;
  if (has_shared) {
    if (!map(&gu.g[1].tmap_b, hidden, L.x8_s, T, H, box_s)) return DWDP_ERR_CUDA;
    gu.g[1].w = shared->w13; gu.g[1].s = shared->s13; gu.g[1].row_scale = nullptr;
    gu.g[1].out = act_blk ? static_cast<void*>(ws + L.h8_s) : static_cast<void*>(h_s);
    gu.g[1].out_scale = sh_s; gu.g[1].os_ld = T;
    gu.g[1].x_scale = sx_s; gu.g[1].xs_ld = T;
    gu.g[1].K = H; gu.g[1].R = Is; gu.g[1].scale_mode = shared->scale_mode; gu.g[1].box_rows = box_s;
    gu.g[1].mstride = (long long)(H / BK8) * kW8TileBytes; gu.g[1].kstride = kW8TileBytes;
  }
  gu.items = items_gu; gu.n_items = n_items; gu.st = st; gu.cap = L.cap_gu;

  dn.g[0].enabled = N > 0;
  if (N > 0 && !map(&dn.g[0].tmap_b, h_r, L.h8_r, N, I, box_r)) return DWDP_ERR_CUDA;
  dn.g[0].w = routed->w2; dn.g[0].s = routed->s2; dn.g[0].out = weighted_out; dn.g[0].box_rows = box_r;
  dn.g[0].x_scale = sh_r; dn.g[0].xs_ld = N;
  dn.g[0].row_scale = packed_weights; dn.g[0].K = I; dn.g[0].R = H; dn.g[0].scale_mode = routed->scale_mode;
  dn.g[0].mstride = (long long)BM * I; dn.g[0].kstride = kW8TileBytes;
  dn.g[1].enabled = has_shared;
  if (has_shared) {
    if (!map(&dn.g[1].tmap_b, h_s, L.h8_s, T, Is, box_s)) return DWDP_ERR_CUDA;
    dn.g[1].w = shared->w2; dn.g[1].s = shared->s2; dn.g[1].out = shared_out; dn.g[1].box_rows = box_s;
    dn.g[1].x_scale = sh_s; dn.g[1].xs_ld = T;
    dn.g[1].row_scale = shared_gate; dn.g[1].K = Is; dn.g[1].R = H; dn.g[1].scale_mode = shared->scale_mode;
    dn.g[1].mstride = (long long)BM * Is; dn.g[1].kstride = kW8TileBytes;
    dn.g[1].part_stride = (long long)T * H;
  }
  dn.items = items_dn; dn.n_items = n_items + 1; dn.st = st; dn.cap = L.cap_dn;

  const int sms = dwdp_device_sm_count();
  if (sms <= 0) return DWDP_ERR_CUDA;
  const int grid_gu = std::max(1, std::min(sms, L.cap_gu));
  const int grid_dn = std::max(1, std::min(sms, L.cap_dn));
  auto quant_h = [&]() {
    return launch_chained(quant_kernel, dim3(quant_blocks(q_rows)), dim3(kPlanThreads), 0, stream, 1u, qh) ==
                   cudaSuccess
               ? DWDP_OK
               : DWDP_ERR_CUDA;
  };
  int rc;
  if (use_pair_blk) {
    // the gate/up epilogue writes the e4m3 intermediate and its scales: no launch between
    const int grid2 = std::max(2, (sms / 2) * 2);
    rc = launch_gemm_f8x2p<0>(gu, grid2, stream);
    if (rc == DWDP_OK) rc = launch_gemm_f8x2p<1>(dn, grid2, stream);
  } else if (use_pair) {
    const int grid2 = std::max(2, (sms / 2) * 2);
    rc = pair_kps == 2 ? launch_gemm_f8x2<0, 2>(gu, grid2, stream) : launch_gemm_f8x2<0, 1>(gu, grid2, stream);
    if (rc == DWDP_OK) rc = quant_h();
    if (rc == DWDP_OK)
      rc = pair_kps == 2 ? launch_gemm_f8x2<1, 2>(dn, grid2, stream) : launch_gemm_f8x2<1, 1>(dn, grid2, stream);
  } else if (hilo_native) {
    rc = wide ? launch_gemm_f8<0, 2, 128>(gu, grid_gu, stream) : launch_gemm_f8<0, 2, 64>(gu, grid_gu, stream);
    if (rc == DWDP_OK) rc = quant_h();
    if (rc == DWDP_OK) {
      if (wide) rc = pair_dn ? launch_gemm_f8<1, 2, 128>(dn, grid_dn, stream) : launch_gemm_f8<1, 1, 128>(dn, grid_dn, stream);
      else rc = pair_dn ? launch_gemm_f8<1, 2, 64>(dn, grid_dn, stream) : launch_gemm_f8<1, 1, 64>(dn, grid_dn, stream);
    }
  } else if (promote && act_blk) {
    // the gate/up epilogue writes the e4m3 intermediate and its scales: no launch between
    if (wide) {
      rc = launch_gemm_f8p<0, 2, 128, 1>(gu, grid_gu, stream);
      if (rc == DWDP_OK) rc = launch_gemm_f8p<1, 1, 128, 1>(dn, grid_dn, stream);
    } else {
      rc = launch_gemm_f8p<0, 2, 64, 1>(gu, grid_gu, stream);
      if (rc == DWDP_OK)
        rc = pair_dn ? launch_gemm_f8p<1, 2, 64, 1>(dn, grid_dn, stream) : launch_gemm_f8p<1, 1, 64, 1>(dn, grid_dn, stream);
    }
  } else if (promote) {
    rc = launch_gemm_f8p<0, 2, 64, 2>(gu, grid_gu, stream);
    if (rc == DWDP_OK) rc = quant_h();
    if (rc == DWDP_OK)
      rc = pair_dn ? launch_gemm_f8p<1, 2, 64, 2>(dn, grid_dn, stream) : launch_gemm_f8p<1, 1, 64, 2>(dn, grid_dn, stream);
  } else {
    rc = launch_gemm<0>(gu, grid_gu, stream);
    if (rc == DWDP_OK) rc = launch_gemm<1>(dn, grid_dn, stream);
  }
  return rc;
}

// The reference's quantize_activations_blockwise (DWDP/executor/fp8.py:86-115) alone:
// rows of `src` (bf16 [src_rows, K], row r read from row_index[r] when given) -> e4m3
// [rows, K] and fp32 scales [rows][K / 128] (scale_rowmajor) or [K / 128][rows].
extern "C" int dwdp_quantize_activations_launch(const void* src, int64_t src_rows, const int64_t* row_index,
                                                int64_t rows, int K, void* dst, float* scales, int scale_rowmajor,
                                                int* status, cudaStream_t stream) {
  if (rows < 0 || K <= 0 || K % 128 != 0 || rows > INT32_MAX) return DWDP_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DWDP_OK;
  QuantParams q{};
  q.seg[0] = QuantSeg{reinterpret_cast<const __nv_bfloat16*>(src), reinterpret_cast<uint8_t*>(dst), scales,
                      (int)rows, K, row_index, src_rows, scale_rowmajor};
  q.st = reinterpret_cast<DeviceStatus*>(status);
  q.blk = 1;
  q.per_warp = 1;
  return launch_chained(quant_kernel, dim3(quant_blocks_blk(rows * ((K + 511) / 512))), dim3(kPlanThreads), 0,
                        stream, 1u, q) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

#ifdef DWDP_PROFILE_ROLES
// Diagnostic build only: how many two-CTA clusters of the pair kernels can be resident at once.
extern "C" int dwdp_debug_max_pair_clusters(int* hilo, int* blk) {
  auto query = [](auto kfn, int threads, int smem, int* out) {
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -3;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 148);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaOccupancyMaxActiveClusters(out, kfn, &cfg) == cudaSuccess ? 0 : -3;
  };
  using C = dwdp::CfgX2<0, 2>;
  if (query(dwdp::moe_gemm_f8x2_kernel<0, 2>, C::THREADS, C::SMEM_BYTES, hilo) != 0) return -3;
  return query(dwdp::moe_gemm_f8x2p_kernel<0>, dwdp::CfgX2P::THREADS, dwdp::CfgX2P::SMEM_BYTES, blk);
}

extern "C" int dwdp_debug_role_cycles(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, dwdp::g_role_cycles, sizeof(dwdp::g_role_cycles)) == cudaSuccess ? 0 : -3;
}
#endif

// Expert weight store: one-shot quantisation + tiling of expert projections
// into the layout the grouped GEMM streams with single bulk copies.
//
// Quantisation restates DWDP/executor/fp8.py:118-146 (quantize_weights_blockwise:
// scale = max(amax over the 128x128 block, 1e-5) / 448, q = e4m3(w / scale)) and,
// for per-output-channel scales (which the reference has no function for), the
// same rule with the amax taken over one output row. Division is IEEE (rn) and
// the e4m3 conversion rounds to nearest even with saturation, as torch does for
// in-range values, so the quantised bytes equal torch's.
//
// Per-tensor scales (DWDP/executor/fp8.py:45-49, convert_qwen_weights_to_fp8_once
// with a scale_map: scale = max(amax of the whole matrix, 1e-5) / 448) are stored
// per output row like CHANNEL scales, every row of a matrix holding the same value,
// so the GEMMs treat both modes alike.
//
// Tile layout (tile_slot):
//   fp8 : tile (rb, kb) of matrix p at index (rb * P + p) * KB + kb: a row block's tiles of one
//         matrix are contiguous along K, so a GEMM stage can bring two K blocks of a matrix
//         with one bulk copy; the matrices of a row block follow each other.
//   bf16: at index (rb * KB + kb) * P + p: both matrices of one K step side by side (the bf16
//         kernel loads them with one copy).
//   fp8 (all modes): 128 rows x 128 inputs, 128-byte rows in the 128B-swizzled
//                 smem image (16-byte chunk c of row r stored at chunk c ^ (r & 7)):
//                 the e4m3 operand the tcgen05 kind::f8f6f4 MMA reads directly.
//                 A BLOCK128 tile is exactly one scale block.
//   bf16        : 128 rows x 64 inputs, 128-byte rows in the swizzled image.
#include "common.cuh"

namespace dwdp {

constexpr int kTileRows = 128;

__host__ __device__ inline int64_t tile_slot(int rb, int kb, int p, int KB, int P, int dst_dtype) {
  return dst_dtype == DWDP_DTYPE_FP8_E4M3 ? ((int64_t)rb * P + p) * KB + kb : ((int64_t)rb * KB + kb) * P + p;
}

// inputs per tile for a (dtype, scale mode) pair
__host__ __device__ inline int tile_cols(int dst_dtype, int mode) {
  (void)mode;
  return dst_dtype == DWDP_DTYPE_FP8_E4M3 ? 128 : 64;
}

template <typename TS>
__device__ __forceinline__ float ldf(const TS* p, int64_t i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

struct MatPtrs {
  const void* p[2];
};

__host__ __device__ inline bool row_scaled(int mode) {
  return mode == DWDP_SCALE_CHANNEL || mode == DWDP_SCALE_TENSOR;
}

// amax per output row (CHANNEL, TENSOR) or per 128x128 block (BLOCK128) -> scales.
// TENSOR writes the raw row amax; tensor_scale_kernel then folds the rows.
template <typename TS>
__global__ void scale_kernel(MatPtrs src, int R, int C, int mode, float* __restrict__ scales) {
  const int p = blockIdx.z;
  const TS* w = reinterpret_cast<const TS*>(src.p[p]);
  __shared__ float red[32];
  float m = 0.f;
  int64_t out_index;
  if (row_scaled(mode)) {
    const int r = blockIdx.x;
    for (int c = threadIdx.x; c < C; c += blockDim.x) m = fmaxf(m, fabsf(ldf(w, (int64_t)r * C + c)));
    out_index = (int64_t)p * R + r;
  } else {
    const int rb = blockIdx.x, cb = blockIdx.y;
    for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
      const int r = rb * 128 + i / 128, c = cb * 128 + i % 128;
      m = fmaxf(m, fabsf(ldf(w, (int64_t)r * C + c)));
    }
    out_index = ((int64_t)p * (R / 128) + rb) * (C / 128) + cb;
  }
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a = fmaxf(a, red[i]);
    scales[out_index] = mode == DWDP_SCALE_TENSOR ? a : __fdiv_rn(fmaxf(a, 1e-5f), 448.0f);
  }
}

// TENSOR: matrix p's row amaxes [p][R] -> max over the rows, scale written to every row.
__global__ void tensor_scale_kernel(int R, float* __restrict__ scales) {
  float* s = scales + (int64_t)blockIdx.x * R;
  __shared__ float red[32];
  float m = 0.f;
  for (int r = threadIdx.x; r < R; r += blockDim.x) m = fmaxf(m, s[r]);
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float a = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a = fmaxf(a, red[i]);
  __syncthreads();
  const float sc = __fdiv_rn(fmaxf(a, 1e-5f), 448.0f);
  for (int r = threadIdx.x; r < R; r += blockDim.x) s[r] = sc;
}

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// one CTA per tile, one thread per tile row
template <typename TS>
__global__ void __launch_bounds__(128)
tile_kernel(MatPtrs src, int R, int C, int P, int dst_dtype, int mode,
            const float* __restrict__ scales, uint8_t* __restrict__ dst) {
  const int kb = blockIdx.x, rb = blockIdx.y, p = blockIdx.z;
  const int kTileCols = tile_cols(dst_dtype, mode);
  const int KB = C / kTileCols;
  const int r = threadIdx.x;
  const int grow = rb * kTileRows + r;
  const TS* w = reinterpret_cast<const TS*>(src.p[p]);
  const int64_t tile_index = tile_slot(rb, kb, p, KB, P, dst_dtype);
  const int64_t row_base = (int64_t)grow * C + kb * kTileCols;
  if (dst_dtype == DWDP_DTYPE_FP8_E4M3) {
    float s;
    if (row_scaled(mode)) s = scales[(int64_t)p * R + grow];
    else s = scales[((int64_t)p * (R / 128) + rb) * (C / 128) + (kb * kTileCols) / 128];
    uint8_t* out = dst + tile_index * (kTileRows * kTileCols) + r * kTileCols;
    for (int c = 0; c < kTileCols; c += 16) {
      alignas(16) uint8_t b[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) b[j] = to_e4m3(__fdiv_rn(ldf(w, row_base + c + j), s));
      *reinterpret_cast<uint4*>(out + (((c >> 4) ^ (r & 7)) << 4)) = *reinterpret_cast<uint4*>(b);
    }
  } else {
    uint8_t* out = dst + tile_index * (kTileRows * kTileCols * 2) + r * 128;
    for (int chunk = 0; chunk < 8; ++chunk) {
      alignas(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __float2bfloat16_rn(ldf(w, row_base + chunk * 8 + j));
      *reinterpret_cast<uint4*>(out + ((chunk ^ (r & 7)) << 4)) = *reinterpret_cast<uint4*>(v);
    }
  }
}

__global__ void __launch_bounds__(128)
untile_kernel(const uint8_t* __restrict__ tiles, const float* __restrict__ scales, int R, int C,
              int P, int dst_dtype, int mode, float* __restrict__ out) {
  const int kb = blockIdx.x, rb = blockIdx.y, p = blockIdx.z;
  const int kTileCols = tile_cols(dst_dtype, mode);
  const int KB = C / kTileCols;
  const int r = threadIdx.x;
  const int grow = rb * kTileRows + r;
  const int64_t tile_index = tile_slot(rb, kb, p, KB, P, dst_dtype);
  float* o = out + ((int64_t)p * R + grow) * C + kb * kTileCols;
  if (dst_dtype == DWDP_DTYPE_FP8_E4M3) {
    float s;
    if (row_scaled(mode)) s = scales[(int64_t)p * R + grow];
    else s = scales[((int64_t)p * (R / 128) + rb) * (C / 128) + (kb * kTileCols) / 128];
    const uint8_t* in = tiles + tile_index * (kTileRows * kTileCols) + r * kTileCols;
    for (int c = 0; c < kTileCols; ++c) {
      __nv_fp8_e4m3 q;
      q.__x = in[(((c >> 4) ^ (r & 7)) << 4) | (c & 15)];
      o[c] = float(q) * s;
    }
  } else {
    const uint8_t* in = tiles + tile_index * (kTileRows * kTileCols * 2) + r * 128;
    for (int c = 0; c < kTileCols; ++c) {
      const int chunk = c >> 3;
      const __nv_bfloat16* v =
          reinterpret_cast<const __nv_bfloat16*>(in + ((chunk ^ (r & 7)) << 4)) + (c & 7);
      o[c] = __bfloat162float(*v);
    }
  }
}

}  // namespace dwdp

using namespace dwdp;

extern "C" size_t dwdp_packed_weight_bytes(int rows, int cols, int num_mats, int dst_dtype) {
  const size_t elems = (size_t)rows * cols * num_mats;
  return dst_dtype == DWDP_DTYPE_FP8_E4M3 ? elems : elems * 2;
}

extern "C" size_t dwdp_packed_scale_floats(int rows, int cols, int num_mats, int scale_mode) {
  if (scale_mode == DWDP_SCALE_CHANNEL || scale_mode == DWDP_SCALE_TENSOR) return (size_t)num_mats * rows;
  if (scale_mode == DWDP_SCALE_BLOCK128) return (size_t)num_mats * (rows / 128) * (cols / 128);
  return 0;
}

static bool pack_args_ok(int rows, int cols, int P, int dst_dtype, int mode) {
  if (rows <= 0 || cols <= 0 || (rows % 128) != 0 || (cols % 128) != 0) return false;
  if (P != 1 && P != 2) return false;
  if (dst_dtype == DWDP_DTYPE_FP8_E4M3)
    return mode == DWDP_SCALE_CHANNEL || mode == DWDP_SCALE_BLOCK128 || mode == DWDP_SCALE_TENSOR;
  if (dst_dtype == DWDP_DTYPE_BF16) return mode == DWDP_SCALE_NONE;
  return false;
}

extern "C" int dwdp_pack_launch(const void* const* src_mats, int src_dtype, int rows, int cols,
                                int P, int dst_dtype, int mode, void* dst, float* scales,
                                cudaStream_t stream) {
  if (!pack_args_ok(rows, cols, P, dst_dtype, mode) || src_mats == nullptr || dst == nullptr)
    return DWDP_ERR_INVALID_ARGUMENT;
  if (dst_dtype == DWDP_DTYPE_FP8_E4M3 && scales == nullptr) return DWDP_ERR_INVALID_ARGUMENT;
  MatPtrs m{};
  for (int p = 0; p < P; ++p) m.p[p] = src_mats[p];
  const dim3 tgrid(cols / tile_cols(dst_dtype, mode), rows / kTileRows, P);
#define DWDP_PACK(TS)                                                                          \
  do {                                                                                         \
    if (dst_dtype == DWDP_DTYPE_FP8_E4M3) {                                                    \
      if (row_scaled(mode))                                                                    \
        scale_kernel<TS><<<dim3(rows, 1, P), 256, 0, stream>>>(m, rows, cols, mode, scales);   \
      else                                                                                     \
        scale_kernel<TS><<<dim3(rows / 128, cols / 128, P), 256, 0, stream>>>(m, rows, cols,   \
                                                                              mode, scales);   \
      if (mode == DWDP_SCALE_TENSOR) tensor_scale_kernel<<<P, 1024, 0, stream>>>(rows, scales); \
    }                                                                                          \
    tile_kernel<TS><<<tgrid, 128, 0, stream>>>(m, rows, cols, P, dst_dtype, mode, scales,      \
                                               (uint8_t*)dst);                                 \
  } while (0)
  if (src_dtype == DWDP_DTYPE_F32) DWDP_PACK(float);
  else if (src_dtype == DWDP_DTYPE_BF16) DWDP_PACK(__nv_bfloat16);
  else return DWDP_ERR_UNSUPPORTED;
#undef DWDP_PACK
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

extern "C" int dwdp_unpack_launch(const void* tiles, const float* scales, int rows, int cols,
                                  int P, int dst_dtype, int mode, float* out,
                                  cudaStream_t stream) {
  if (!pack_args_ok(rows, cols, P, dst_dtype, mode)) return DWDP_ERR_INVALID_ARGUMENT;
  const dim3 tgrid(cols / tile_cols(dst_dtype, mode), rows / kTileRows, P);
  untile_kernel<<<tgrid, 128, 0, stream>>>((const uint8_t*)tiles, scales, rows, cols, P,
                                           dst_dtype, mode, out);
  return cudaGetLastError() == cudaSuccess ? DWDP_OK : DWDP_ERR_CUDA;
}

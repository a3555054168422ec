// Expert-parallel (EP) decode exchange over NVLink peer memory: token rows travel to the
// rank that owns their expert and the weighted results travel back, with no host
// synchronisation and no collective library call on the data path.
//
// Replaces the reference's decode EP path (DWDP/adapters/qwen15_moe.py:164-243): there, a
// bincount + all_to_all_single of counts, a host .tolist(), three all_to_all_single of
// rows / expert ids, a Python loop over local experts and a reverse all_to_all_single.
// Ownership is the reference's: owner(e) = min(e / ceil(E / world), world - 1).
//
// Every rank holds one EP buffer (layout below, byte offsets from EpLayout) mapped into
// every other rank through CUDA IPC; `peers[r]` is rank r's buffer as seen from here
// (peers[rank] = the local buffer). Per forward:
//   ep_send    rows x[t] for slot (t, k) -> peers[owner].recv_x[rank][pos], with their
//              (expert, flat slot id, routing weight); each CTA then raises every owner's
//              recv_arrive[rank] by one (system-scope release).
//   ep_plan    (owner) waits until every source's CTAs arrived, resets the counters,
//              counting-sorts the received rows by local expert: counts / offsets,
//              source row, routing weight and return address per packed row.
//   ep_gather  packed rows in expert order (the grouped GEMM's packed_hidden).
//   (grouped expert GEMMs, weighted by the routing weight in the down epilogue)
//   ep_return  weighted rows -> peers[src].ret_y[flat slot id]; each CTA raises every
//              source's ret_arrive by one.
//   ep_wait    (source) waits for every owner's CTAs, resets the counter; the merge of
//              ret_y (slot order) + shared expert follows.
// One buffer set suffices: a rank sends the next layer's rows only after it received
// this layer's results from every owner, which each owner returns only after it has
// copied its received rows out (ep_gather) and reset its counters (ep_plan).
// Waits are bounded: on timeout the kernel records DWDP_ERR_DEVICE_TIMEOUT and goes on.
#include "common.cuh"

namespace dwdp {

struct EpLayout {
  int world, rank, H, cap;  // cap = rows one source may send to one owner (T_max * K)
  size_t recv_x, recv_meta, recv_count, recv_arrive, ret_y, ret_arrive, total;
};

struct EpMeta {
  int expert;   // global expert id
  int slot;     // flat slot id t * K + k at the source
  float weight; // routing weight
  int pad;
};

__host__ __device__ inline size_t ep_align(size_t x) { return (x + 255) / 256 * 256; }

__host__ __device__ inline EpLayout ep_layout(int world, int rank, int H, int cap) {
  EpLayout L{world, rank, H, cap, 0, 0, 0, 0, 0, 0, 0};
  size_t o = 0;
  L.recv_x = o;      o = ep_align(o + (size_t)world * cap * H * 2);
  L.recv_meta = o;   o = ep_align(o + (size_t)world * cap * sizeof(EpMeta));
  L.recv_count = o;  o = ep_align(o + (size_t)world * sizeof(int));
  L.recv_arrive = o; o = ep_align(o + (size_t)world * sizeof(int));
  L.ret_y = o;       o = ep_align(o + (size_t)cap * H * 2);
  L.ret_arrive = o;  o = ep_align(o + sizeof(int));
  L.total = o;
  return L;
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= target (about a second at most).
__device__ __forceinline__ bool ep_wait_geq(const int* p, int target) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (ld_acquire_sys(p) >= target) return true;
    __nanosleep(128);
  }
  return false;
}

__device__ __forceinline__ int ep_owner(int e, int E, int world) {
  const int per = (E + world - 1) / world;
  return min(e / per, world - 1);
}

__device__ __forceinline__ uint8_t* peer_base(const unsigned long long* peers, int r) {
  return reinterpret_cast<uint8_t*>(peers[r]);
}

// Warp copy of one H-wide bf16 row (H % 8 == 0), 16 bytes per lane per step.
__device__ __forceinline__ void warp_copy_row(__nv_bfloat16* dst, const __nv_bfloat16* src, int H, int lane) {
  for (int c = lane * 8; c < H; c += 256)
    *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
}

constexpr int kEpThreads = 256;
constexpr int kEpMaxSlots = 2048;  // T * K per rank

// ---------------------------------------------------------------------------
// ep_send: positions by owner (stable in slot order), rows + metadata to the owners.
// Every CTA recomputes the positions (n <= 2048 slots, warp ballots) and copies the
// rows of the slots assigned to its warps.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEpThreads)
ep_send_kernel(const __nv_bfloat16* __restrict__ x, const int64_t* __restrict__ topk_idx,
               const float* __restrict__ topk_w, int T, int K, int E, EpLayout L,
               const unsigned long long* __restrict__ peers, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  __shared__ int s_pos[kEpMaxSlots];
  __shared__ int s_dst[kEpMaxSlots];
  __shared__ int s_warp[kEpThreads / 32][8];
  __shared__ int s_base[8];
  const int n = T * K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 8) s_base[tid] = 0;
  __syncthreads();
  for (int c0 = 0; c0 < n; c0 += kEpThreads) {
    const int i = c0 + tid;
    int d = -1;
    if (i < n) {
      const int e = (int)topk_idx[i];
      if (e < 0 || e >= E) {
        record_error(st, DWDP_ERR_DEVICE_BOUNDS, 500, i);
      } else {
        d = ep_owner(e, E, L.world);
      }
      s_dst[i] = d;
    }
    for (int r = 0; r < L.world; ++r) {
      const unsigned m = __ballot_sync(0xffffffffu, d == r);
      if (lane == 0) s_warp[warp][r] = __popc(m);
      __syncthreads();
      if (d == r) {
        int before = s_base[r];
        for (int w = 0; w < warp; ++w) before += s_warp[w][r];
        s_pos[i] = before + __popc(m & ((1u << lane) - 1u));
      }
      __syncthreads();
      if (tid == 0) {
        int tot = 0;
        for (int w = 0; w < kEpThreads / 32; ++w) tot += s_warp[w][r];
        s_base[r] += tot;
      }
      __syncthreads();
    }
  }
  // rows: warp-granular over the grid
  const int gw = blockIdx.x * (kEpThreads / 32) + warp, nw = gridDim.x * (kEpThreads / 32);
  for (int i = gw; i < n; i += nw) {
    const int d = s_dst[i];
    if (d < 0) continue;
    const int pos = s_pos[i];
    if (pos >= L.cap) {
      if (lane == 0) record_error(st, DWDP_ERR_CAPACITY, 501, pos);
      continue;
    }
    uint8_t* base = peer_base(peers, d);
    const size_t row = (size_t)L.rank * L.cap + pos;
    warp_copy_row(reinterpret_cast<__nv_bfloat16*>(base + L.recv_x) + row * L.H, x + (size_t)(i / K) * L.H, L.H,
                  lane);
    if (lane == 0) {
      EpMeta m{(int)topk_idx[i], i, topk_w[i], 0};
      reinterpret_cast<EpMeta*>(base + L.recv_meta)[row] = m;
    }
  }
  if (blockIdx.x == 0 && tid < L.world)
    reinterpret_cast<int*>(peer_base(peers, tid) + L.recv_count)[L.rank] = min(s_base[tid], L.cap);
  __threadfence_system();
  __syncthreads();
  if (tid < L.world) atomicAdd_system(reinterpret_cast<int*>(peer_base(peers, tid) + L.recv_arrive) + L.rank, 1);
}

// ---------------------------------------------------------------------------
// ep_plan (one CTA, owner side): wait for every source, reset the counters, then the
// counting sort of the received rows by local expert (slot order inside an expert is
// not significant: a row's result does not depend on its neighbours).
// Outputs: counts[El], offsets[El + 1] (int64), packed_src[p] (row of recv_x),
// packed_w[p], ret_addr[p] = src * 2^20 + slot, total[0].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
ep_plan_kernel(EpLayout L, int E, int expert_lo, int El, int send_ctas, int64_t* __restrict__ counts,
               int64_t* __restrict__ offsets, int* __restrict__ packed_src, float* __restrict__ packed_w,
               int* __restrict__ ret_addr, int* __restrict__ total, DeviceStatus* st, uint8_t* own) {
  griddep_launch();
  griddep_wait();
  __shared__ int s_cnt[256], s_off[257], s_fill[256], s_rows[8];
  const int tid = threadIdx.x;
  int* arrive = reinterpret_cast<int*>(own + L.recv_arrive);
  if (tid < L.world) {
    if (!ep_wait_geq(arrive + tid, send_ctas)) record_error(st, DWDP_ERR_DEVICE_TIMEOUT, 510, tid);
    __threadfence_system();
    // Subtract this layer's arrivals instead of storing 0: after a timeout, CTAs that arrive
    // late bring the counter back to 0 rather than satisfying the next layer's wait early.
    atomicSub(arrive + tid, send_ctas);
    s_rows[tid] = min(ld_acquire_sys(reinterpret_cast<int*>(own + L.recv_count) + tid), L.cap);
  }
  if (tid < El) s_cnt[tid] = 0, s_fill[tid] = 0;
  __syncthreads();
  const EpMeta* meta = reinterpret_cast<const EpMeta*>(own + L.recv_meta);
  const int rows_all = L.world * L.cap;
  for (int r = tid; r < rows_all; r += blockDim.x) {
    const int s = r / L.cap, i = r % L.cap;
    if (i < s_rows[s]) {
      const int le = meta[r].expert - expert_lo;
      if (le >= 0 && le < El) atomicAdd(&s_cnt[le], 1);
      else record_error(st, DWDP_ERR_DEVICE_BOUNDS, 511, meta[r].expert);
    }
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < El; ++e) {
      s_off[e] = acc;
      acc += s_cnt[e];
    }
    s_off[El] = acc;
    total[0] = acc;
  }
  __syncthreads();
  if (tid < El) counts[tid] = s_cnt[tid];
  if (tid <= El) offsets[tid] = s_off[tid];
  for (int r = tid; r < rows_all; r += blockDim.x) {
    const int s = r / L.cap, i = r % L.cap;
    if (i < s_rows[s]) {
      const EpMeta m = meta[r];
      const int le = m.expert - expert_lo;
      if (le < 0 || le >= El) continue;
      const int p = s_off[le] + atomicAdd(&s_fill[le], 1);
      packed_src[p] = r;
      packed_w[p] = m.weight;
      ret_addr[p] = (s << 20) | m.slot;
    }
  }
}

// packed_hidden[p] = recv_x[packed_src[p]] for p < total.
__global__ void __launch_bounds__(kEpThreads)
ep_gather_kernel(EpLayout L, const uint8_t* own, const int* __restrict__ packed_src, const int* __restrict__ total,
                 __nv_bfloat16* __restrict__ packed) {
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const int n = total[0];
  const __nv_bfloat16* rx = reinterpret_cast<const __nv_bfloat16*>(own + L.recv_x);
  for (int p = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); p < n; p += gridDim.x * (kEpThreads / 32))
    warp_copy_row(packed + (size_t)p * L.H, rx + (size_t)packed_src[p] * L.H, L.H, lane);
}

// weighted[p] -> peers[src].ret_y[slot]; then every CTA raises every source's ret_arrive.
// The return address comes from a peer's metadata: source and slot are bounds-checked.
__global__ void __launch_bounds__(kEpThreads)
ep_return_kernel(EpLayout L, const __nv_bfloat16* __restrict__ weighted, const int* __restrict__ ret_addr,
                 const int* __restrict__ total, const unsigned long long* __restrict__ peers, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const int n = total[0];
  for (int p = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); p < n; p += gridDim.x * (kEpThreads / 32)) {
    const int a = ret_addr[p];
    const int s = a >> 20, slot = a & 0xFFFFF;
    if (s < 0 || s >= L.world || slot >= L.cap) {
      if (lane == 0) record_error(st, DWDP_ERR_DEVICE_BOUNDS, 530, a);
      continue;
    }
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peer_base(peers, s) + L.ret_y) + (size_t)slot * L.H;
    warp_copy_row(dst, weighted + (size_t)p * L.H, L.H, lane);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < L.world) atomicAdd_system(reinterpret_cast<int*>(peer_base(peers, threadIdx.x) + L.ret_arrive), 1);
}

// Source side: wait for every owner's return CTAs, reset.
__global__ void ep_wait_kernel(EpLayout L, uint8_t* own, int expected, DeviceStatus* st) {
  griddep_launch();
  griddep_wait();
  if (threadIdx.x == 0) {
    int* c = reinterpret_cast<int*>(own + L.ret_arrive);
    if (!ep_wait_geq(c, expected)) record_error(st, DWDP_ERR_DEVICE_TIMEOUT, 520, ld_acquire_sys(c));
    __threadfence_system();
    atomicSub(c, expected);  // late arrivals after a timeout cancel out instead of carrying over
  }
}

}  // namespace dwdp

using namespace dwdp;

extern "C" size_t dwdp_ep_buffer_bytes(int world, int hidden_size, int capacity) {
  if (world <= 0 || world > 8 || hidden_size <= 0 || capacity <= 0) return 0;
  return ep_layout(world, 0, hidden_size, capacity).total;
}

// The grid sizes below are part of the protocol (arrival counts): every rank uses the same.
constexpr int kEpSendCtas = 16;
constexpr int kEpReturnCtas = 16;

extern "C" int dwdp_ep_dispatch_launch(const void* x, const int64_t* topk_idx, const float* topk_w, int T, int K,
                                       int E, int world, int rank, int H, int cap,
                                       const unsigned long long* peers, int* status, cudaStream_t stream) {
  // T == 0 still launches: the owners count one arrival per send CTA of every source
  if (T < 0 || T * K > kEpMaxSlots || world > 8 || H % 8) return DWDP_ERR_UNSUPPORTED;
  const EpLayout L = ep_layout(world, rank, H, cap);
  return launch_chained(ep_send_kernel, dim3(kEpSendCtas), dim3(kEpThreads), 0, stream, 1u,
                        (const __nv_bfloat16*)x, topk_idx, topk_w, T, K, E, L, peers,
                        reinterpret_cast<DeviceStatus*>(status)) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

extern "C" int dwdp_ep_plan_launch(void* own, int world, int rank, int H, int cap, int E, int expert_lo, int El,
                                   int64_t* counts, int64_t* offsets, int* packed_src, float* packed_w,
                                   int* ret_addr, int* total, void* packed_hidden, int* status,
                                   cudaStream_t stream) {
  if (El <= 0 || El > 256 || world > 8) return DWDP_ERR_UNSUPPORTED;
  const EpLayout L = ep_layout(world, rank, H, cap);
  DeviceStatus* st = reinterpret_cast<DeviceStatus*>(status);
  if (launch_chained(ep_plan_kernel, dim3(1), dim3(1024), 0, stream, 1u, L, E, expert_lo, El, kEpSendCtas, counts,
                     offsets, packed_src, packed_w, ret_addr, total, st, (uint8_t*)own) != cudaSuccess)
    return DWDP_ERR_CUDA;
  return launch_chained(ep_gather_kernel, dim3(2 * dwdp_device_sm_count()), dim3(kEpThreads), 0, stream, 1u, L,
                        (const uint8_t*)own, (const int*)packed_src, (const int*)total,
                        (__nv_bfloat16*)packed_hidden) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

extern "C" int dwdp_ep_combine_launch(void* own, int world, int rank, int H, int cap, const void* weighted,
                                      const int* ret_addr, const int* total, const unsigned long long* peers,
                                      int* status, cudaStream_t stream) {
  const EpLayout L = ep_layout(world, rank, H, cap);
  if (launch_chained(ep_return_kernel, dim3(kEpReturnCtas), dim3(kEpThreads), 0, stream, 1u, L,
                     (const __nv_bfloat16*)weighted, ret_addr, total, peers,
                     reinterpret_cast<DeviceStatus*>(status)) != cudaSuccess)
    return DWDP_ERR_CUDA;
  return launch_chained(ep_wait_kernel, dim3(1), dim3(32), 0, stream, 1u, L, (uint8_t*)own, world * kEpReturnCtas,
                        reinterpret_cast<DeviceStatus*>(status)) == cudaSuccess
             ? DWDP_OK
             : DWDP_ERR_CUDA;
}

extern "C" size_t dwdp_ep_ret_offset(int world, int hidden_size, int capacity) {
  return ep_layout(world, 0, hidden_size, capacity).ret_y;
}

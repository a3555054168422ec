// DWDP communication engine (host C++, CUDA runtime API only).
//
// Replaces the reference's native engine (DWDP/communication/
// communication_engine.cpp, buffers.cu, ipc.cu, events.cu, topology.cpp,
// transfer_scheduler.cpp, communication_policy.cpp; bound in bindings.cpp:32-111)
// with a design for one 8xB200 NVSwitch box:
//
//  * An expert is one contiguous slab (weights + scales), so a remote expert is
//    ONE peer copy. Copies run on greatest-priority non-blocking streams owned by
//    the engine (experts spread round-robin over kCopyStreams so several copy
//    engines work at once) and take no SMs from the GEMMs.
//  * Staging is N buffers of fixed slots (slot = largest registered slab); a
//    remote expert has the same slot index in every buffer, so the caller's
//    pointer arrays for buffer b are computed once.
//  * prefetch(ids, buffer) issues the copies for one layer with a rotated start
//    (by device id) so 8 ranks do not all read the same peer first, then records
//    one event per buffer; wait(buffer, stream) makes the CALLER's stream wait on
//    it (the reference waited on an engine-private stream).
//  * IPC export returns the allocation handle plus the pointer's offset inside
//    the allocation (the reference exported the handle of the first parameter
//    and ignored the allocator's sub-allocation offset).
//  * Transfer scheduling (priority queue, coalescing, two retries) and the path
//    policy are plain host code with their own C ABI, testable without a GPU.
#include <cstdlib>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "dwdp_b200.h"
#include "prefetch_plan.h"

namespace {

int set_error(const char* what, cudaError_t e);

struct EngineExpert {
  int id = -1;
  bool remote = false;
  const void* src = nullptr;  // local slab or opened peer pointer
  size_t bytes = 0;
  int slot = -1;              // staging slot (remote experts only)
  int owner_device = -1;
};

struct IpcMapping {
  void* base = nullptr;
  int refs = 0;
};

}  // namespace

constexpr int kCopyStreams = 4;  // copies of one prefetch spread over this many streams

struct dwdp_engine {
  int device = 0;
  size_t slot_bytes = 0;
  int num_buffers = 0;
  size_t buffer_bytes = 0;
  std::vector<void*> buffers;
  std::vector<cudaEvent_t> ready;     // copies of buffer b done
  std::vector<int> buffer_valid;      // buffer b holds the last prefetch
  cudaStream_t copy_stream = nullptr;  // stream 0 of copy_streams
  std::vector<cudaStream_t> copy_streams;       // experts spread round-robin (several copy engines)
  std::vector<cudaEvent_t> stream_done;         // per copy stream, joined into ready[b]
  std::map<int, EngineExpert> experts;
  std::map<std::string, IpcMapping> ipc;  // handle bytes -> opened base
  int next_slot = 0;
  unsigned long long bytes_copied = 0;
  unsigned long long copies_issued = 0;
  // DWDP_COPY_SM: SM copy kernels instead of the copy engines (env DWDP_COPY_SM_CTAS=n at
  // creation, or dwdp_engine_set_copy_mode)
  int copy_mode = DWDP_COPY_ENGINE;
  int copy_ctas = 148;
  std::mutex mu;
};

namespace {

thread_local std::string g_engine_error;

int fail(int code, const std::string& msg) {
  g_engine_error = msg;
  return code;
}

int set_error(const char* what, cudaError_t e) {
  g_engine_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return DWDP_ERR_CUDA;
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev_);
    ok_ = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() { cudaSetDevice(prev_); }
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = false;
};

using PFN_getAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_getAddressRange address_range_fn() {
  static PFN_getAddressRange fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_getAddressRange>(p);
  }
  return fn;
}

}  // namespace

extern "C" const char* dwdp_engine_last_error(void) { return g_engine_error.c_str(); }

// ----------------------------------------------------------------------------- topology / IPC
extern "C" int dwdp_peer_can_access(int src_device, int dst_device, int* out) {
  if (out == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "peer_can_access: null output");
  if (src_device == dst_device) {
    *out = 1;
    return DWDP_OK;
  }
  int v = 0;
  const cudaError_t e = cudaDeviceCanAccessPeer(&v, dst_device, src_device);
  if (e != cudaSuccess) return set_error("cudaDeviceCanAccessPeer", e);
  *out = v;
  return DWDP_OK;
}

extern "C" int dwdp_export_ipc_handle(const void* device_ptr, void* handle_out, size_t* offset_out) {
  if (device_ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "export_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(device_ptr));
  if (e != cudaSuccess) return set_error("cudaIpcGetMemHandle", e);
  auto fn = address_range_fn();
  if (fn == nullptr) return fail(DWDP_ERR_CUDA, "export_ipc_handle: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
    return fail(DWDP_ERR_CUDA, "export_ipc_handle: cuMemGetAddressRange failed");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<size_t>(device_ptr) - static_cast<size_t>(base);
  return DWDP_OK;
}

extern "C" size_t dwdp_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

// Open another process's allocation (its export_ipc_handle blob) and return the device
// address of `offset` inside it; dwdp_ipc_close takes the base that was returned in *base_out.
extern "C" int dwdp_ipc_open(const void* handle, size_t offset, void** base_out, void** ptr_out) {
  if (handle == nullptr || base_out == nullptr || ptr_out == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error("cudaIpcOpenMemHandle", e);
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return DWDP_OK;
}

extern "C" int dwdp_ipc_close(void* base) {
  if (base == nullptr) return DWDP_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? DWDP_OK : set_error("cudaIpcCloseMemHandle", e);
}

// ----------------------------------------------------------------------------- engine
extern "C" int dwdp_engine_create(int device_id, size_t slot_bytes, int num_slots, int num_buffers,
                                  dwdp_engine** out) {
  if (out == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "engine_create: null output");
  *out = nullptr;
  if (num_buffers < 1 || num_buffers > 4 || num_slots < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "engine_create: num_buffers must be 1..4, num_slots >= 0");
  DeviceGuard guard(device_id);
  if (!guard.ok()) return fail(DWDP_ERR_CUDA, "engine_create: cannot select device");
  auto eng = std::make_unique<dwdp_engine>();
  eng->device = device_id;
  eng->slot_bytes = (slot_bytes + 255) & ~size_t(255);
  eng->num_buffers = num_buffers;
  eng->buffer_bytes = eng->slot_bytes * (size_t)num_slots;
  int lo = 0, hi = 0;
  cudaError_t e = cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if (e != cudaSuccess) return set_error("cudaDeviceGetStreamPriorityRange", e);
  int n_streams = kCopyStreams;
  if (const char* v = std::getenv("DWDP_COPY_STREAMS")) n_streams = std::max(1, std::min(8, std::atoi(v)));  // tuning
  if (const char* v = std::getenv("DWDP_COPY_SM_CTAS")) {  // tuning: SM copies with n CTAs
    const int n = std::atoi(v);
    if (n > 0) {
      eng->copy_mode = DWDP_COPY_SM;
      eng->copy_ctas = n;
    }
  }
  for (int i = 0; i < n_streams; ++i) {
    cudaStream_t cs;
    e = cudaStreamCreateWithPriority(&cs, cudaStreamNonBlocking, hi);  // greatest priority
    if (e != cudaSuccess) return set_error("cudaStreamCreateWithPriority", e);
    eng->copy_streams.push_back(cs);
    cudaEvent_t ev;
    cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    eng->stream_done.push_back(ev);
  }
  eng->copy_stream = eng->copy_streams[0];
  for (int b = 0; b < num_buffers; ++b) {
    void* p = nullptr;
    if (eng->buffer_bytes > 0) {
      e = cudaMalloc(&p, eng->buffer_bytes);
      if (e != cudaSuccess) {
        for (void* q : eng->buffers) cudaFree(q);
        for (auto cs : eng->copy_streams) cudaStreamDestroy(cs);
        for (auto ev : eng->stream_done) cudaEventDestroy(ev);
        return set_error("cudaMalloc(staging)", e);
      }
    }
    eng->buffers.push_back(p);
    cudaEvent_t ev;
    cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    eng->ready.push_back(ev);
    eng->buffer_valid.push_back(0);
  }
  *out = eng.release();
  return DWDP_OK;
}

extern "C" int dwdp_engine_destroy(dwdp_engine* eng) {
  if (eng == nullptr) return DWDP_OK;
  {
    DeviceGuard guard(eng->device);
    for (auto cs : eng->copy_streams) cudaStreamSynchronize(cs);
    for (void* p : eng->buffers)
      if (p) cudaFree(p);
    for (auto ev : eng->ready) cudaEventDestroy(ev);
    for (auto& kv : eng->ipc)
      if (kv.second.base) cudaIpcCloseMemHandle(kv.second.base);
    for (auto cs : eng->copy_streams) cudaStreamDestroy(cs);
    for (auto ev : eng->stream_done) cudaEventDestroy(ev);
  }
  delete eng;
  return DWDP_OK;
}

extern "C" int dwdp_engine_register_local(dwdp_engine* eng, int expert_id, const void* ptr, size_t bytes) {
  if (eng == nullptr || ptr == nullptr || expert_id < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "register_local: bad argument");
  std::lock_guard<std::mutex> lock(eng->mu);
  EngineExpert x;
  x.id = expert_id;
  x.remote = false;
  x.src = ptr;
  x.bytes = bytes;
  x.owner_device = eng->device;
  eng->experts[expert_id] = x;
  return DWDP_OK;
}

extern "C" int dwdp_engine_register_ipc(dwdp_engine* eng, int expert_id, const void* handle, size_t offset,
                                        size_t bytes, int owner_device) {
  if (eng == nullptr || handle == nullptr || expert_id < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "register_ipc: bad argument");
  if (bytes > eng->slot_bytes)
    return fail(DWDP_ERR_CAPACITY, "register_ipc: expert of " + std::to_string(bytes) +
                                       " bytes exceeds the staging slot of " + std::to_string(eng->slot_bytes));
  std::lock_guard<std::mutex> lock(eng->mu);
  if ((size_t)(eng->next_slot + 1) * eng->slot_bytes > eng->buffer_bytes && eng->experts.count(expert_id) == 0)
    return fail(DWDP_ERR_CAPACITY, "register_ipc: staging buffers have no free slot");
  DeviceGuard guard(eng->device);
  const std::string key(reinterpret_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
  auto it = eng->ipc.find(key);
  if (it == eng->ipc.end()) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error("cudaIpcOpenMemHandle", e);
    it = eng->ipc.emplace(key, IpcMapping{base, 0}).first;
  }
  it->second.refs++;
  EngineExpert x;
  auto prev = eng->experts.find(expert_id);
  x.slot = (prev != eng->experts.end() && prev->second.remote) ? prev->second.slot : eng->next_slot++;
  x.id = expert_id;
  x.remote = true;
  x.src = static_cast<const char*>(it->second.base) + offset;
  x.bytes = bytes;
  x.owner_device = owner_device;
  eng->experts[expert_id] = x;
  return DWDP_OK;
}

// Register a remote expert by a pointer this process can already address
// (same-process multi-GPU with peer access); used where IPC is unnecessary.
extern "C" int dwdp_engine_register_peer(dwdp_engine* eng, int expert_id, const void* peer_ptr, size_t bytes,
                                         int owner_device) {
  if (eng == nullptr || peer_ptr == nullptr || expert_id < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "register_peer: bad argument");
  if (bytes > eng->slot_bytes) return fail(DWDP_ERR_CAPACITY, "register_peer: expert exceeds the staging slot");
  std::lock_guard<std::mutex> lock(eng->mu);
  auto prev = eng->experts.find(expert_id);
  const bool had_slot = prev != eng->experts.end() && prev->second.remote;
  if (!had_slot && (size_t)(eng->next_slot + 1) * eng->slot_bytes > eng->buffer_bytes)
    return fail(DWDP_ERR_CAPACITY, "register_peer: staging buffers have no free slot");
  EngineExpert x;
  x.slot = had_slot ? prev->second.slot : eng->next_slot++;
  x.id = expert_id;
  x.remote = true;
  x.src = peer_ptr;
  x.bytes = bytes;
  x.owner_device = owner_device;
  eng->experts[expert_id] = x;
  return DWDP_OK;
}

namespace {

struct PlannedCopy {
  const char* src;
  char* dst;
  size_t bytes;
};

// Issue `copies` into staging `buffer` in list order, after the work already queued on
// `after_stream`: copy k goes to copy stream k % streams (copy engines), or the list runs
// as SM copy kernels of up to DWDP_COPY_LIST_MAX copies on stream 0. The copy streams then
// join into stream 0 and one event marks the buffer ready. Caller holds eng->mu.
int issue_copies(dwdp_engine* eng, const std::vector<PlannedCopy>& copies, int buffer, void* after_stream) {
  cudaError_t e;
  if (after_stream != nullptr) {
    // the buffer may still be read by earlier work on the caller's stream
    cudaEvent_t dep;
    e = cudaEventCreateWithFlags(&dep, cudaEventDisableTiming);
    if (e != cudaSuccess) return set_error("cudaEventCreate", e);
    cudaEventRecord(dep, reinterpret_cast<cudaStream_t>(after_stream));
    for (auto cs : eng->copy_streams) cudaStreamWaitEvent(cs, dep, 0);
    cudaEventDestroy(dep);
  }
  if (eng->copy_mode == DWDP_COPY_SM) {
    dwdp_copy_list list;
    list.n = 0;
    for (size_t j = 0; j <= copies.size(); ++j) {
      if (list.n == DWDP_COPY_LIST_MAX || (j == copies.size() && list.n > 0)) {
        const int rc = dwdp_peer_copy_sm(&list, eng->copy_ctas, eng->copy_streams[0]);
        if (rc != DWDP_OK) return fail(rc, "prefetch: SM copy launch failed");
        eng->copies_issued += 1;
        list.n = 0;
      }
      if (j == copies.size()) break;
      list.src[list.n] = copies[j].src;
      list.dst[list.n] = copies[j].dst;
      list.bytes[list.n] = copies[j].bytes;
      ++list.n;
      eng->bytes_copied += copies[j].bytes;
    }
  } else {
    for (size_t k = 0; k < copies.size(); ++k) {
      e = cudaMemcpyAsync(copies[k].dst, copies[k].src, copies[k].bytes, cudaMemcpyDeviceToDevice,
                          eng->copy_streams[k % eng->copy_streams.size()]);
      if (e != cudaSuccess) return set_error("cudaMemcpyAsync(prefetch)", e);
      eng->copies_issued += 1;
      eng->bytes_copied += copies[k].bytes;
    }
  }
  for (size_t i = 1; i < eng->copy_streams.size(); ++i) {
    cudaEventRecord(eng->stream_done[i], eng->copy_streams[i]);
    cudaStreamWaitEvent(eng->copy_streams[0], eng->stream_done[i], 0);
  }
  e = cudaEventRecord(eng->ready[buffer], eng->copy_streams[0]);
  if (e != cudaSuccess) return set_error("cudaEventRecord", e);
  eng->buffer_valid[buffer] = 1;
  return DWDP_OK;
}

char* staging_slot(dwdp_engine* eng, const EngineExpert* x, int buffer) {
  return static_cast<char*>(eng->buffers[buffer]) + (size_t)x->slot * eng->slot_bytes;
}

}  // namespace

extern "C" int dwdp_engine_prefetch(dwdp_engine* eng, const int* expert_ids, int n, int buffer,
                                    void* after_stream) {
  if (eng == nullptr || (n > 0 && expert_ids == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "prefetch: bad argument");
  if (buffer < 0 || buffer >= eng->num_buffers) return fail(DWDP_ERR_INVALID_ARGUMENT, "prefetch: bad buffer");
  std::lock_guard<std::mutex> lock(eng->mu);
  DeviceGuard guard(eng->device);
  std::vector<const EngineExpert*> todo;
  for (int i = 0; i < n; ++i) {
    auto it = eng->experts.find(expert_ids[i]);
    if (it == eng->experts.end()) return fail(DWDP_ERR_NOT_FOUND, "prefetch: unknown expert " + std::to_string(expert_ids[i]));
    if (it->second.remote) todo.push_back(&it->second);
  }
  // Order and granularity: dwdp_plan::plan_prefetch (prefetch_plan.h). With DWDP_PREFETCH_SLICE_MB
  // = s > 0 every expert moves as s-MiB slices (the reference's 2 MiB scheme); otherwise each
  // owner's contiguous experts move as ~DWDP_PREFETCH_COALESCE_MB-MiB pieces (default 64; 0 = one
  // copy per expert): per-copy rates on B200 grow with the copy (8.65 MB 492 GB/s, 44 MB 670,
  // 176 MB 721). SM copies always move whole experts.
  static const size_t slice = [] {
    const char* v = getenv("DWDP_PREFETCH_SLICE_MB");
    return v != nullptr ? (size_t)atoi(v) << 20 : (size_t)0;
  }();
  static const size_t coalesce = [] {
    const char* v = getenv("DWDP_PREFETCH_COALESCE_MB");
    return v != nullptr ? (size_t)atoi(v) << 20 : (size_t)64 << 20;
  }();
  const bool sm = eng->copy_mode == DWDP_COPY_SM;
  std::vector<dwdp_plan::Expert> remote;
  remote.reserve(todo.size());
  for (const EngineExpert* x : todo)
    remote.push_back(dwdp_plan::Expert{x->owner_device, static_cast<const char*>(x->src), staging_slot(eng, x, buffer),
                                       x->bytes});
  const auto plan = dwdp_plan::plan_prefetch(remote, eng->device, sm ? 0 : slice, sm ? 0 : coalesce);
  std::vector<PlannedCopy> copies;
  copies.reserve(plan.size());
  for (const auto& c : plan) copies.push_back(PlannedCopy{c.src, c.dst, c.bytes});
  return issue_copies(eng, copies, buffer, after_stream);
}

extern "C" int dwdp_engine_prefetch_slices(dwdp_engine* eng, const dwdp_copy_slice* slices, int n, int buffer,
                                           void* after_stream) {
  if (eng == nullptr || (n > 0 && slices == nullptr) || n < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "prefetch_slices: bad argument");
  if (buffer < 0 || buffer >= eng->num_buffers)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "prefetch_slices: bad buffer");
  std::lock_guard<std::mutex> lock(eng->mu);
  DeviceGuard guard(eng->device);
  std::vector<PlannedCopy> copies;
  copies.reserve((size_t)n);
  for (int i = 0; i < n; ++i) {
    const dwdp_copy_slice& sl = slices[i];
    auto it = eng->experts.find(sl.expert_id);
    if (it == eng->experts.end())
      return fail(DWDP_ERR_NOT_FOUND, "prefetch_slices: unknown expert " + std::to_string(sl.expert_id));
    const EngineExpert* x = &it->second;
    if (sl.start > x->bytes || sl.bytes > x->bytes - sl.start)
      return fail(DWDP_ERR_INVALID_ARGUMENT, "prefetch_slices: slice beyond expert " + std::to_string(sl.expert_id));
    if (!x->remote || sl.bytes == 0) continue;  // local experts are read in place
    copies.push_back(PlannedCopy{static_cast<const char*>(x->src) + sl.start, staging_slot(eng, x, buffer) + sl.start,
                                 (size_t)sl.bytes});
  }
  return issue_copies(eng, copies, buffer, after_stream);
}

extern "C" int dwdp_engine_set_copy_mode(dwdp_engine* eng, int mode, int ctas) {
  if (eng == nullptr || (mode != DWDP_COPY_ENGINE && mode != DWDP_COPY_SM) || ctas <= 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "set_copy_mode: bad argument");
  std::lock_guard<std::mutex> lock(eng->mu);
  eng->copy_mode = mode;
  eng->copy_ctas = ctas;
  return DWDP_OK;
}

extern "C" int dwdp_engine_wait(dwdp_engine* eng, int buffer, void* stream) {
  if (eng == nullptr || buffer < 0 || buffer >= eng->num_buffers)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "wait: bad argument");
  if (!eng->buffer_valid[buffer]) return fail(DWDP_ERR_STATE, "wait: buffer was never prefetched");
  const cudaError_t e = cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), eng->ready[buffer], 0);
  return e == cudaSuccess ? DWDP_OK : set_error("cudaStreamWaitEvent", e);
}

extern "C" int dwdp_engine_resident_pointer(dwdp_engine* eng, int expert_id, int buffer, void** out) {
  if (eng == nullptr || out == nullptr || buffer < 0 || buffer >= eng->num_buffers)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "resident_pointer: bad argument");
  std::lock_guard<std::mutex> lock(eng->mu);
  auto it = eng->experts.find(expert_id);
  if (it == eng->experts.end()) return fail(DWDP_ERR_NOT_FOUND, "resident_pointer: unknown expert " + std::to_string(expert_id));
  if (!it->second.remote) {
    *out = const_cast<void*>(it->second.src);
  } else {
    *out = static_cast<char*>(eng->buffers[buffer]) + (size_t)it->second.slot * eng->slot_bytes;
  }
  return DWDP_OK;
}

extern "C" int dwdp_engine_is_remote(dwdp_engine* eng, int expert_id, int* out) {
  if (eng == nullptr || out == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "is_remote: bad argument");
  std::lock_guard<std::mutex> lock(eng->mu);
  auto it = eng->experts.find(expert_id);
  if (it == eng->experts.end()) return fail(DWDP_ERR_NOT_FOUND, "is_remote: unknown expert");
  *out = it->second.remote ? 1 : 0;
  return DWDP_OK;
}

extern "C" int dwdp_engine_release(dwdp_engine* eng, int expert_id) {
  if (eng == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "release: null engine");
  std::lock_guard<std::mutex> lock(eng->mu);
  auto it = eng->experts.find(expert_id);
  if (it == eng->experts.end()) return fail(DWDP_ERR_NOT_FOUND, "release: unknown expert");
  eng->experts.erase(it);
  return DWDP_OK;
}

extern "C" int dwdp_engine_synchronize(dwdp_engine* eng) {
  if (eng == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "synchronize: null engine");
  DeviceGuard guard(eng->device);
  for (auto cs : eng->copy_streams) {
    const cudaError_t e = cudaStreamSynchronize(cs);
    if (e != cudaSuccess) return set_error("cudaStreamSynchronize", e);
  }
  return DWDP_OK;
}

extern "C" int dwdp_engine_stats(dwdp_engine* eng, unsigned long long* bytes_copied,
                                 unsigned long long* copies_issued, void** copy_stream) {
  if (eng == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "stats: null engine");
  std::lock_guard<std::mutex> lock(eng->mu);
  if (bytes_copied) *bytes_copied = eng->bytes_copied;
  if (copies_issued) *copies_issued = eng->copies_issued;
  if (copy_stream) *copy_stream = eng->copy_stream;
  return DWDP_OK;
}

// ----------------------------------------------------------------------------- path policy
// Same decision table as DWDP/communication/communication_policy.cpp:5-17 (the
// drop-in contract): an expert already staged/active is local; one with an IPC
// handle goes through IPC; another GPU's expert with peer access is a P2P read;
// otherwise a staged copy. Path codes follow CommunicationPath (bindings.cpp:94-99).
extern "C" int dwdp_policy_decide(int local_gpu, int owner_gpu, int resident_state, int has_ipc_handle,
                                  int peer_access) {
  if (resident_state == DWDP_RESIDENT_STAGED || resident_state == DWDP_RESIDENT_ACTIVE) return DWDP_PATH_LOCAL;
  if (has_ipc_handle) return DWDP_PATH_IPC;
  if (owner_gpu != local_gpu && peer_access) return DWDP_PATH_P2P;
  return DWDP_PATH_COPY;
}

// ----------------------------------------------------------------------------- transfer scheduler
// Priority queue of expert transfers (higher priority first, FIFO among equals),
// coalescing repeated submissions of a queued/running expert, at most two retries
// of a retryable failure, cancellation of queued transfers only, and a bounded
// blocking take(). Mirrors TransferScheduler's contract (bindings.cpp:84-92).
struct dwdp_sched {
  struct Task {
    int id;
    int priority;
    unsigned long long seq;
    int state;
    int retries;
  };
  struct Order {
    bool operator()(const Task* a, const Task* b) const {
      return a->priority == b->priority ? a->seq > b->seq : a->priority < b->priority;
    }
  };
  std::mutex mu;
  std::condition_variable cv;
  std::priority_queue<Task*, std::vector<Task*>, Order> q;
  std::unordered_map<int, std::unique_ptr<Task>> live;  // queued or running
  std::unordered_map<int, int> final_state;             // last terminal state per expert
  std::vector<std::unique_ptr<Task>> cancelled;         // still referenced by the queue
  unsigned long long seq = 0;
  bool closed = false;
};

extern "C" int dwdp_sched_create(dwdp_sched** out) {
  if (out == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "sched_create: null output");
  *out = new dwdp_sched();
  return DWDP_OK;
}

extern "C" int dwdp_sched_destroy(dwdp_sched* s) {
  delete s;
  return DWDP_OK;
}

extern "C" int dwdp_sched_submit(dwdp_sched* s, int expert_id, int priority) {
  if (s == nullptr || expert_id < 0) return fail(DWDP_ERR_INVALID_ARGUMENT, "submit: invalid expert id");
  std::lock_guard<std::mutex> lock(s->mu);
  if (s->closed) return fail(DWDP_ERR_STATE, "submit: scheduler closed");
  if (s->live.count(expert_id)) return DWDP_OK;  // coalesced with the pending transfer
  auto t = std::make_unique<dwdp_sched::Task>(dwdp_sched::Task{expert_id, priority, s->seq++, DWDP_TRANSFER_QUEUED, 0});
  s->q.push(t.get());
  s->live[expert_id] = std::move(t);
  s->final_state.erase(expert_id);
  s->cv.notify_one();
  return DWDP_OK;
}

// Pops the next transfer into *expert_id (state RUNNING). *expert_id = -1 when the
// scheduler is closed and drained; DWDP_ERR_DEVICE_TIMEOUT after timeout_ms.
extern "C" int dwdp_sched_take(dwdp_sched* s, int timeout_ms, int* expert_id) {
  if (s == nullptr || expert_id == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "take: bad argument");
  std::unique_lock<std::mutex> lock(s->mu);
  for (;;) {
    while (!s->q.empty() && s->q.top()->state == DWDP_TRANSFER_CANCELLED) s->q.pop();
    if (!s->q.empty()) break;
    if (s->closed) {
      *expert_id = -1;
      return DWDP_OK;
    }
    if (!s->cv.wait_for(lock, std::chrono::milliseconds(timeout_ms < 0 ? 0 : timeout_ms), [&] {
          while (!s->q.empty() && s->q.top()->state == DWDP_TRANSFER_CANCELLED) s->q.pop();
          return s->closed || !s->q.empty();
        }))
      return fail(DWDP_ERR_DEVICE_TIMEOUT, "take: no transfer within the timeout");
  }
  dwdp_sched::Task* t = s->q.top();
  s->q.pop();
  t->state = DWDP_TRANSFER_RUNNING;
  *expert_id = t->id;
  return DWDP_OK;
}

static int sched_finish(dwdp_sched* s, int expert_id, int state) {
  auto it = s->live.find(expert_id);
  s->final_state[expert_id] = state;
  s->live.erase(it);
  return DWDP_OK;
}

extern "C" int dwdp_sched_complete(dwdp_sched* s, int expert_id) {
  if (s == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "complete: null scheduler");
  std::lock_guard<std::mutex> lock(s->mu);
  auto it = s->live.find(expert_id);
  if (it == s->live.end() || it->second->state != DWDP_TRANSFER_RUNNING)
    return fail(DWDP_ERR_STATE, "complete: illegal transfer transition");
  return sched_finish(s, expert_id, DWDP_TRANSFER_COMPLETED);
}

extern "C" int dwdp_sched_fail(dwdp_sched* s, int expert_id, int retryable) {
  if (s == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "fail: null scheduler");
  std::lock_guard<std::mutex> lock(s->mu);
  auto it = s->live.find(expert_id);
  if (it == s->live.end() || it->second->state != DWDP_TRANSFER_RUNNING)
    return fail(DWDP_ERR_STATE, "fail: illegal transfer transition");
  dwdp_sched::Task* t = it->second.get();
  if (retryable && t->retries < 2 && !s->closed) {
    t->retries++;
    t->state = DWDP_TRANSFER_QUEUED;
    s->q.push(t);
    s->cv.notify_one();
    return DWDP_OK;
  }
  return sched_finish(s, expert_id, DWDP_TRANSFER_FAILED);
}

extern "C" int dwdp_sched_cancel(dwdp_sched* s, int expert_id) {
  if (s == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "cancel: null scheduler");
  std::lock_guard<std::mutex> lock(s->mu);
  auto it = s->live.find(expert_id);
  if (it == s->live.end()) return DWDP_OK;
  if (it->second->state != DWDP_TRANSFER_QUEUED)
    return fail(DWDP_ERR_STATE, "cancel: only a queued transfer may be cancelled");
  it->second->state = DWDP_TRANSFER_CANCELLED;  // skipped by take(); the queue drops it lazily
  s->final_state[expert_id] = DWDP_TRANSFER_CANCELLED;
  s->cancelled.push_back(std::move(it->second));  // the heap entry still points at it
  s->live.erase(it);
  return DWDP_OK;
}

extern "C" int dwdp_sched_close(dwdp_sched* s) {
  if (s == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "close: null scheduler");
  std::lock_guard<std::mutex> lock(s->mu);
  s->closed = true;
  s->cv.notify_all();
  return DWDP_OK;
}

extern "C" int dwdp_sched_state(dwdp_sched* s, int expert_id, int* state, int* retries) {
  if (s == nullptr || state == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "state: bad argument");
  std::lock_guard<std::mutex> lock(s->mu);
  auto it = s->live.find(expert_id);
  if (it != s->live.end()) {
    *state = it->second->state;
    if (retries) *retries = it->second->retries;
    return DWDP_OK;
  }
  auto f = s->final_state.find(expert_id);
  if (f == s->final_state.end()) return fail(DWDP_ERR_NOT_FOUND, "state: unknown transfer");
  *state = f->second;
  if (retries) *retries = 0;
  return DWDP_OK;
}

// C ABI entry points (include/dwdp_b200.h): argument validation, the
// thread-local error message, and dispatch to the kernel launchers.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"

extern "C" int dwdp_router_launch(const void*, int, const void*, int, const float*, const void*,
                                  int64_t, int, int, int, float, int, float, float*, float*,
                                  int64_t*, float*, float*, cudaStream_t);
extern "C" int dwdp_dispatch_launch(const int64_t*, const void*, int, int64_t, int, int, int64_t*,
                                    int64_t*, int64_t*, int64_t*, int64_t*, int64_t*, void*,
                                    const void*, int, void*, void*, int*, cudaStream_t);
extern "C" int dwdp_dispatch_noalloc_launch(const int64_t*, const void*, int, int64_t, int, int,
                                            int64_t*, int64_t*, int64_t*, int64_t*, int64_t*,
                                            int64_t*, void*, const void*, int, void*, int*,
                                            cudaStream_t);
extern "C" size_t dwdp_dispatch_noalloc_max_scratch_bytes(void);
extern "C" int dwdp_gather_rows_launch(const void*, const int64_t*, int64_t, int, int64_t, void*, int*,
                                       cudaStream_t);
extern "C" size_t dwdp_dispatch_scratch_bytes(int64_t, int, int);
extern "C" int dwdp_route_dispatch_small_launch(const void*, const void*, const float*, const void*, int64_t, int,
                                                int, int, float, int, float, float*, float*, float*, int64_t*,
                                                float*, float*, int64_t*, int64_t*, int64_t*, int64_t*, int64_t*,
                                                int64_t*, float*, int*, int*, cudaStream_t);
extern "C" int dwdp_quantize_activations_launch(const void*, int64_t, const int64_t*, int64_t, int, void*, float*,
                                                int, int*, cudaStream_t);
extern "C" int dwdp_schedule_launch(const int64_t*, const int64_t*, int, int, int64_t*, int64_t*,
                                    int64_t*, int64_t*, int64_t*, int64_t*, int64_t*, cudaStream_t);
extern "C" int dwdp_pack_launch(const void* const*, int, int, int, int, int, int, void*, float*,
                                cudaStream_t);
extern "C" int dwdp_unpack_launch(const void*, const float*, int, int, int, int, int, float*,
                                  cudaStream_t);
extern "C" size_t dwdp_moe_workspace_bytes_impl(int64_t, int, int, int, int, int);
extern "C" int dwdp_moe_experts_launch(const dwdp_expert_group*, const dwdp_expert_group*,
                                       const void*, const int64_t*, const void*, int64_t, int, const int64_t*,
                                       const int64_t*, const float*, const float*, void*, void*,
                                       void*, size_t, int*, int, cudaStream_t);
extern "C" size_t dwdp_moe_shared_workspace_bytes_impl(int64_t, int, int);
extern "C" int dwdp_tensor_list_build_launch(const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                                             const int64_t*, int, const dwdp_expert_group*,
                                             const dwdp_tensor_list_bases*, int64_t, int64_t*, int64_t*, int*,
                                             cudaStream_t);
extern "C" int dwdp_merge_launch(const void*, const int64_t*, const void*, int, const float*, int64_t, int, int,
                                 void*, int, int*, cudaStream_t);

extern "C" int dwdp_add_rmsnorm_launch(void*, const void*, const void*, int64_t, int, float, void*, cudaStream_t);
extern "C" int dwdp_rope_append_launch(const void*, const void*, const int32_t*, const int32_t*, int, int, int, int, int,
                                       int, float, void*, void*, void*, int*, cudaStream_t);
extern "C" size_t dwdp_paged_attention_workspace_bytes_impl(int, int, int);
extern "C" int dwdp_paged_attention_launch(const void*, const void*, const void*, const int32_t*, const int32_t*, int, int,
                                           int, int, int, int, int, int, float, void*, void*, int*,
                                           cudaStream_t);

extern "C" size_t dwdp_ep_buffer_bytes(int, int, int);
extern "C" size_t dwdp_ep_ret_offset(int, int, int);
extern "C" int dwdp_ep_dispatch_launch(const void*, const int64_t*, const float*, int, int, int, int, int, int, int,
                                       const unsigned long long*, int*, cudaStream_t);
extern "C" int dwdp_ep_plan_launch(void*, int, int, int, int, int, int, int, int64_t*, int64_t*, int*, float*, int*,
                                   int*, void*, int*, cudaStream_t);
extern "C" int dwdp_ep_combine_launch(void*, int, int, int, int, const void*, const int*, const int*,
                                      const unsigned long long*, int*, cudaStream_t);

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check(int rc, const char* what) {
  if (rc == DWDP_OK) return rc;
  if (rc == DWDP_ERR_CUDA) {
    cudaError_t e = cudaGetLastError();
    return fail(rc, "%s: CUDA error %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  }
  if (g_last_error.empty()) return fail(rc, "%s failed with status %d", what, rc);
  return rc;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

extern "C" int dwdp_version(void) { return 100; }

extern "C" const char* dwdp_last_error(void) { return g_last_error.c_str(); }

extern "C" int dwdp_router_topk(const void* hidden, int hidden_dtype, const void* weight,
                                int weight_dtype, const float* bias, const void* shared_gate_weight,
                                int64_t num_tokens, int hidden_size, int num_experts, int top_k,
                                float score_scale, int renormalize, float eps, float* logits,
                                float* probs, int64_t* topk_idx, float* topk_weights,
                                float* shared_gate, int* status, void* stream) {
  g_last_error.clear();
  (void)status;
  if (num_tokens < 0 || hidden_size <= 0) return fail(DWDP_ERR_INVALID_ARGUMENT, "router: bad sizes");
  if (num_experts <= 0 || num_experts > 256)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "router: num_experts must be in [1, 256], got %d", num_experts);
  if (top_k <= 0 || top_k > 16 || top_k > num_experts)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "router: top_k must be in [1, min(16, E)], got %d", top_k);
  if (!(score_scale > 0.f) || !(eps > 0.f))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "router: score_scale and eps must be > 0");
  if (num_tokens > 0 && (hidden == nullptr || weight == nullptr || topk_idx == nullptr || topk_weights == nullptr ||
                         logits == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "router: null pointer");
  if (shared_gate_weight != nullptr && shared_gate == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "router: shared_gate output required with a gate weight");
  return check(dwdp_router_launch(hidden, hidden_dtype, weight, weight_dtype, bias, shared_gate_weight,
                                  num_tokens, hidden_size, num_experts, top_k, score_scale, renormalize,
                                  eps, logits, probs, topk_idx, topk_weights, shared_gate,
                                  as_stream(stream)),
               "router");
}

extern "C" int dwdp_dispatch(const int64_t* topk_idx, const void* topk_weights, int weight_dtype,
                             int64_t num_tokens, int top_k, int num_experts, int64_t* counts,
                             int64_t* offsets, int64_t* perm, int64_t* inv, int64_t* ids, int64_t* tok,
                             void* packed_weights, const void* hidden, int hidden_size,
                             void* packed_hidden, void* scratch, int* status, void* stream) {
  g_last_error.clear();
  if (num_experts <= 0 || num_experts > 1024)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch: num_experts must be in [1, 1024], got %d", num_experts);
  if (top_k <= 0 || num_tokens < 0) return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch: bad top_k/num_tokens");
  if (num_tokens * top_k > ((int64_t)1 << 31) - 1)
    return fail(DWDP_ERR_CAPACITY, "dispatch: more than 2^31 assignments");
  if (counts == nullptr || offsets == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch: null counts/offsets");
  if (num_tokens > 0 && (topk_idx == nullptr || topk_weights == nullptr || perm == nullptr || inv == nullptr ||
                         ids == nullptr || tok == nullptr || packed_weights == nullptr || scratch == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch: null pointer");
  if (packed_hidden != nullptr && (hidden == nullptr || hidden_size <= 0))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch: packed_hidden needs hidden and hidden_size");
  return check(dwdp_dispatch_launch(topk_idx, topk_weights, weight_dtype, num_tokens, top_k, num_experts,
                                    counts, offsets, perm, inv, ids, tok, packed_weights, hidden,
                                    hidden_size, packed_hidden, scratch, status, as_stream(stream)),
               "dispatch");
}

extern "C" int dwdp_dispatch_noalloc(const int64_t* topk_idx, const void* topk_weights, int weight_dtype,
                                     int64_t num_tokens, int top_k, int num_experts, int64_t* counts,
                                     int64_t* offsets, int64_t* perm, int64_t* inv, int64_t* ids,
                                     int64_t* tok, void* packed_weights, const void* hidden,
                                     int hidden_size, void* packed_hidden, int* status, void* stream) {
  g_last_error.clear();
  if (num_experts <= 0 || num_experts > 1024)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch_noalloc: num_experts must be in [1, 1024], got %d",
                num_experts);
  if (top_k <= 0 || num_tokens < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch_noalloc: bad top_k/num_tokens");
  if (num_tokens * top_k > ((int64_t)1 << 31) - 1)
    return fail(DWDP_ERR_CAPACITY, "dispatch_noalloc: more than 2^31 assignments");
  const size_t need = dwdp_dispatch_scratch_bytes(num_tokens, top_k, num_experts) - 256;
  const size_t have = dwdp_dispatch_noalloc_max_scratch_bytes();
  if (need > have)
    return fail(DWDP_ERR_CAPACITY,
                "dispatch_noalloc: ceil(T*K/256)*E*4 = %zu bytes of histogram scratch exceed the fixed "
                "%zu-byte buffer; use dwdp_dispatch with caller-provided scratch",
                need, have);
  if (counts == nullptr || offsets == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch_noalloc: null counts/offsets");
  if (num_tokens > 0 && (topk_idx == nullptr || topk_weights == nullptr || perm == nullptr || inv == nullptr ||
                         ids == nullptr || tok == nullptr || packed_weights == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch_noalloc: null pointer");
  if (packed_hidden != nullptr && (hidden == nullptr || hidden_size <= 0))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "dispatch_noalloc: packed_hidden needs hidden and hidden_size");
  return check(dwdp_dispatch_noalloc_launch(topk_idx, topk_weights, weight_dtype, num_tokens, top_k,
                                            num_experts, counts, offsets, perm, inv, ids, tok,
                                            packed_weights, hidden, hidden_size, packed_hidden, status,
                                            as_stream(stream)),
               "dispatch_noalloc");
}

extern "C" int dwdp_gather_rows(const void* hidden, const int64_t* token_index, int64_t num_rows, int hidden_size,
                                int64_t num_tokens, void* packed, int* status, void* stream) {
  g_last_error.clear();
  if (num_rows < 0 || hidden_size <= 0 || num_tokens < 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "gather_rows: bad sizes");
  if (num_rows > 0 && (hidden == nullptr || token_index == nullptr || packed == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "gather_rows: null pointer");
  return check(dwdp_gather_rows_launch(hidden, token_index, num_rows, hidden_size, num_tokens, packed, status,
                                       as_stream(stream)),
               "gather_rows");
}

extern "C" int dwdp_route_dispatch_small(const void* hidden, const void* weight, const float* bias,
                                         const void* shared_gate_weight, int64_t num_tokens, int hidden_size,
                                         int num_experts, int top_k, float score_scale, int renormalize, float eps,
                                         float* logits, float* gate_logit, float* probs, int64_t* topk_idx,
                                         float* topk_weights, float* shared_gate, int64_t* counts, int64_t* offsets,
                                         int64_t* perm, int64_t* inv, int64_t* ids, int64_t* tok,
                                         float* packed_weights, int* ticket, int* status, void* stream) {
  g_last_error.clear();
  if (num_tokens <= 0 || top_k <= 0 || num_tokens * top_k > 256 || num_experts <= 0 || num_experts > 256 ||
      top_k > 16 || top_k > num_experts || hidden_size <= 0 || hidden_size % 8 != 0)
    return fail(DWDP_ERR_UNSUPPORTED, "route_dispatch_small: needs 0 < T*K <= 256, E <= 256, K <= 16, H %% 8 == 0");
  if (hidden == nullptr || weight == nullptr || logits == nullptr || topk_idx == nullptr ||
      topk_weights == nullptr || counts == nullptr || offsets == nullptr || perm == nullptr || inv == nullptr ||
      ids == nullptr || tok == nullptr || packed_weights == nullptr || ticket == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "route_dispatch_small: null pointer");
  if (renormalize < 0 || renormalize > 2) return fail(DWDP_ERR_INVALID_ARGUMENT, "route_dispatch_small: bad renormalize");
  return check(dwdp_route_dispatch_small_launch(hidden, weight, bias, shared_gate_weight, num_tokens, hidden_size,
                                                num_experts, top_k, score_scale, renormalize, eps, logits, gate_logit,
                                                probs, topk_idx, topk_weights, shared_gate, counts, offsets, perm, inv,
                                                ids, tok, packed_weights, ticket, status, as_stream(stream)),
               "route_dispatch_small");
}

extern "C" int dwdp_quantize_activations_blockwise(const void* src, int64_t src_rows, const int64_t* row_index,
                                                   int64_t rows, int cols, void* dst, float* scales,
                                                   int scale_layout, int* status, void* stream) {
  g_last_error.clear();
  if (rows < 0 || src_rows < 0 || cols <= 0 || cols % 128 != 0 || rows > INT32_MAX)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "quantize_activations: rows >= 0 and cols a positive multiple of 128");
  if (scale_layout != 0 && scale_layout != 1)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "quantize_activations: scale_layout must be 0 or 1");
  if (row_index == nullptr && rows > src_rows)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "quantize_activations: more rows than the source holds");
  if (rows > 0 && (src == nullptr || dst == nullptr || scales == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "quantize_activations: null pointer");
  return check(dwdp_quantize_activations_launch(src, src_rows, row_index, rows, cols, dst, scales,
                                                scale_layout == 0 ? 1 : 0, status, as_stream(stream)),
               "quantize_activations");
}

extern "C" int dwdp_schedule(const int64_t* counts, const int64_t* offsets, int num_experts,
                             int stream_count, int64_t* expert_queue, int64_t* starts, int64_t* ends,
                             int64_t* active_counts, int64_t* priority, int64_t* stream_ids,
                             int64_t* num_active, void* stream) {
  g_last_error.clear();
  if (num_experts <= 0 || stream_count <= 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "schedule: num_experts and stream_count must be > 0");
  return check(dwdp_schedule_launch(counts, offsets, num_experts, stream_count, expert_queue, starts, ends,
                                    active_counts, priority, stream_ids, num_active, as_stream(stream)),
               "schedule");
}

extern "C" int dwdp_pack_weights(const void* const* src_mats, int src_dtype, int rows, int cols,
                                 int num_mats, int dst_dtype, int scale_mode, void* dst_tiles,
                                 float* dst_scales, void* stream) {
  g_last_error.clear();
  if (rows <= 0 || cols <= 0 || rows % 128 || cols % 128)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "pack_weights: rows (%d) and cols (%d) must be positive multiples of 128",
                rows, cols);
  return check(dwdp_pack_launch(src_mats, src_dtype, rows, cols, num_mats, dst_dtype, scale_mode, dst_tiles,
                                dst_scales, as_stream(stream)),
               "pack_weights");
}

extern "C" int dwdp_unpack_weights(const void* tiles, const float* scales, int rows, int cols, int num_mats,
                                   int dst_dtype, int scale_mode, float* out, void* stream) {
  g_last_error.clear();
  return check(dwdp_unpack_launch(tiles, scales, rows, cols, num_mats, dst_dtype, scale_mode, out,
                                  as_stream(stream)),
               "unpack_weights");
}

extern "C" size_t dwdp_moe_workspace_bytes(int64_t num_tokens, int top_k, int num_experts,
                                           int intermediate_size, int shared_intermediate_size) {
  // The hidden size enters only through the tile count of the down projection;
  // size for the largest supported hidden size (8192) to stay an upper bound.
  return dwdp_moe_workspace_bytes_impl(num_tokens, top_k, num_experts, 8192, intermediate_size,
                                       shared_intermediate_size);
}

namespace {
int moe_experts_checked(const dwdp_expert_group* routed, const dwdp_expert_group* shared,
                        const void* packed_hidden, const int64_t* packed_tok, const void* hidden,
                        int64_t num_tokens, int top_k, const int64_t* counts, const int64_t* offsets,
                        const float* packed_weights, const float* shared_gate, void* weighted_out,
                        void* shared_out, void* workspace, size_t workspace_bytes, int* status, void* stream) {
  g_last_error.clear();
  if (routed == nullptr) return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: routed group is required");
  if (routed->hidden_size <= 0 || routed->hidden_size > 8192)
    return fail(DWDP_ERR_UNSUPPORTED, "moe_experts: hidden_size must be in (0, 8192]");
  if (routed->hidden_size % 128 || routed->intermediate_size <= 0 || routed->intermediate_size % 128 ||
      (shared && (shared->intermediate_size <= 0 || shared->intermediate_size % 128)))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: hidden/intermediate sizes must be multiples of 128");
  if (routed->weight_dtype == DWDP_DTYPE_FP8_E4M3 && routed->scale_mode != DWDP_SCALE_CHANNEL &&
      routed->scale_mode != DWDP_SCALE_BLOCK128 && routed->scale_mode != DWDP_SCALE_TENSOR)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: fp8 weights need a CHANNEL, BLOCK128 or TENSOR scale mode");
  if (routed->act_quant != DWDP_ACT_HILO && routed->act_quant != DWDP_ACT_BLOCK128)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: act_quant must be DWDP_ACT_HILO or DWDP_ACT_BLOCK128");
  if (shared != nullptr && (shared->num_experts != 1 || shared->hidden_size != routed->hidden_size ||
                            shared->weight_dtype != routed->weight_dtype ||
                            shared->scale_mode != routed->scale_mode))
    return fail(DWDP_ERR_INVALID_ARGUMENT,
                "moe_experts: shared group must hold one expert of the routed hidden size, weight dtype and "
                "scale mode");
  if (top_k <= 0 || num_tokens < 0) return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: bad top_k/num_tokens");
  if (num_tokens > 0 && (counts == nullptr || offsets == nullptr || weighted_out == nullptr ||
                         packed_weights == nullptr || (packed_hidden == nullptr && packed_tok == nullptr)))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: null pointer");
  if (packed_tok != nullptr && hidden == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: packed token indices need hidden");
  if (shared != nullptr && (hidden == nullptr || shared_out == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_experts: shared group needs hidden and shared_out");
  const size_t need = dwdp_moe_workspace_bytes(num_tokens, top_k, routed->num_experts,
                                               routed->intermediate_size,
                                               shared ? shared->intermediate_size : 0);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(DWDP_ERR_CAPACITY, "moe_experts: workspace of %zu bytes < required %zu", workspace_bytes, need);
  return check(dwdp_moe_experts_launch(routed, shared, packed_hidden, packed_tok, hidden, num_tokens, top_k,
                                       counts, offsets, packed_weights, shared_gate, weighted_out, shared_out,
                                       workspace, workspace_bytes, status, 0, as_stream(stream)),
               "moe_experts");
}
}  // namespace

extern "C" int dwdp_moe_experts(const dwdp_expert_group* routed, const dwdp_expert_group* shared,
                                const void* packed_hidden, const void* hidden, int64_t num_tokens, int top_k,
                                const int64_t* counts, const int64_t* offsets, const float* packed_weights,
                                const float* shared_gate, void* weighted_out, void* shared_out, void* workspace,
                                size_t workspace_bytes, int* status, void* stream) {
  return moe_experts_checked(routed, shared, packed_hidden, nullptr, hidden, num_tokens, top_k, counts, offsets,
                             packed_weights, shared_gate, weighted_out, shared_out, workspace, workspace_bytes,
                             status, stream);
}

extern "C" int dwdp_moe_experts_indexed(const dwdp_expert_group* routed, const dwdp_expert_group* shared,
                                        const int64_t* packed_token_indices, const void* hidden,
                                        int64_t num_tokens, int top_k, const int64_t* counts,
                                        const int64_t* offsets, const float* packed_weights,
                                        const float* shared_gate, void* weighted_out, void* shared_out,
                                        void* workspace, size_t workspace_bytes, int* status, void* stream) {
  return moe_experts_checked(routed, shared, nullptr, packed_token_indices, hidden, num_tokens, top_k, counts,
                             offsets, packed_weights, shared_gate, weighted_out, shared_out, workspace,
                             workspace_bytes, status, stream);
}

extern "C" int dwdp_merge(const void* weighted, const int64_t* inv, const void* shared_out, int shared_parts,
                          int64_t num_tokens, int top_k, int hidden_size, void* out, int out_dtype,
                          void* stream) {
  g_last_error.clear();
  if (top_k <= 0 || top_k > 16) return fail(DWDP_ERR_INVALID_ARGUMENT, "merge: top_k must be in [1, 16]");
  if (hidden_size <= 0 || hidden_size % 8)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "merge: hidden_size must be a positive multiple of 8");
  if (shared_out != nullptr && (shared_parts < 1 || shared_parts > 64))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "merge: shared_parts must be in [1, 64]");
  return check(dwdp_merge_launch(weighted, inv, shared_out, shared_parts, nullptr, num_tokens, top_k, hidden_size,
                                 out, out_dtype, nullptr, as_stream(stream)),
               "merge");
}

extern "C" int dwdp_merge_gated(const void* weighted, const int64_t* inv, const void* shared_out, int shared_parts,
                                const float* shared_gate, int64_t num_tokens, int top_k, int hidden_size, void* out,
                                int out_dtype, void* stream) {
  g_last_error.clear();
  if (top_k <= 0 || top_k > 16) return fail(DWDP_ERR_INVALID_ARGUMENT, "merge: top_k must be in [1, 16]");
  if (hidden_size <= 0 || hidden_size % 8)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "merge: hidden_size must be a positive multiple of 8");
  if (shared_out == nullptr || shared_gate == nullptr || shared_parts < 1 || shared_parts > 8)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "merge_gated: needs shared_out, shared_gate and 1..8 shared parts");
  return check(dwdp_merge_launch(weighted, inv, shared_out, shared_parts, shared_gate, num_tokens, top_k, hidden_size,
                                 out, out_dtype, nullptr, as_stream(stream)),
               "merge_gated");
}

extern "C" size_t dwdp_moe_shared_workspace_bytes(int64_t num_tokens, int hidden_size, int shared_intermediate_size) {
  return dwdp_moe_shared_workspace_bytes_impl(num_tokens, hidden_size, shared_intermediate_size);
}

extern "C" int dwdp_moe_shared_expert(const dwdp_expert_group* shared, const void* hidden, int64_t num_tokens,
                                      const float* shared_gate, void* shared_out, void* workspace,
                                      size_t workspace_bytes, int* status, void* stream) {
  g_last_error.clear();
  if (shared == nullptr || hidden == nullptr || shared_out == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_shared_expert: shared group, hidden and shared_out are required");
  if (shared->num_experts != 1 || shared->hidden_size <= 0 || shared->hidden_size > 8192 ||
      shared->hidden_size % 128 || shared->intermediate_size <= 0 || shared->intermediate_size % 128)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_shared_expert: one expert, sizes multiples of 128, hidden <= 8192");
  if (num_tokens < 0) return fail(DWDP_ERR_INVALID_ARGUMENT, "moe_shared_expert: bad num_tokens");
  const size_t need = dwdp_moe_shared_workspace_bytes_impl(num_tokens, shared->hidden_size, shared->intermediate_size);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(DWDP_ERR_CAPACITY, "moe_shared_expert: workspace of %zu bytes < required %zu", workspace_bytes, need);
  return check(dwdp_moe_experts_launch(shared, shared, nullptr, nullptr, hidden, num_tokens, 1, nullptr, nullptr,
                                       nullptr, shared_gate, nullptr, shared_out, workspace, workspace_bytes, status, 1,
                                       as_stream(stream)),
               "moe_shared_expert");
}

// --------------------------------------------------------------------------- TensorList
extern "C" int dwdp_tensor_list_build(const int64_t* expert_queue, const int64_t* expert_starts,
                                      const int64_t* expert_counts, const int64_t* priorities,
                                      const int64_t* stream_ids, int plan_len, const dwdp_expert_group* experts,
                                      const dwdp_tensor_list_bases* bases, const dwdp_tensor_list* tl,
                                      int64_t* meta, int* status, void* stream) {
  g_last_error.clear();
  if (experts == nullptr || bases == nullptr || tl == nullptr || meta == nullptr || tl->fields == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "tensor_list_build: null argument");
  if (plan_len < 0 || (plan_len > 0 && (expert_queue == nullptr || expert_starts == nullptr ||
                                        expert_counts == nullptr)))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "tensor_list_build: plan rows missing");
  if (tl->capacity <= 0 || tl->capacity > 1024)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "tensor_list_build: capacity must be in [1, 1024]");
  if (experts->w13 == nullptr || experts->w2 == nullptr || experts->num_experts <= 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "tensor_list_build: expert pointer arrays missing");
  return check(dwdp_tensor_list_build_launch(expert_queue, expert_starts, expert_counts, priorities, stream_ids,
                                             plan_len, experts, bases, tl->capacity, tl->fields, meta, status,
                                             as_stream(stream)),
               "tensor_list_build");
}

extern "C" int dwdp_grouped_moe(const dwdp_tensor_list* tl, const dwdp_expert_group* shared,
                                const int64_t* packed_token_indices, const void* hidden, int64_t num_tokens,
                                int top_k, const float* packed_weights, const float* shared_gate,
                                void* weighted_out, void* shared_out, void* workspace, size_t workspace_bytes,
                                int* status, void* stream) {
  g_last_error.clear();
  if (tl == nullptr || tl->fields == nullptr || tl->capacity <= 0 || tl->capacity > 1024)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "grouped_moe: TensorList with 1..1024 entries required");
  // The TensorList's own rows are the expert group: entry i is "expert" i.
  const int64_t cap = tl->capacity;
  dwdp_expert_group g{};
  g.num_experts = (int)cap;
  g.hidden_size = tl->hidden_size;
  g.intermediate_size = tl->intermediate_size;
  g.weight_dtype = tl->weight_dtype;
  g.scale_mode = tl->scale_mode;
  g.act_quant = tl->act_quant;
  g.w13 = reinterpret_cast<const void* const*>(tl->fields + DWDP_TL_GATE_WEIGHT_PTRS * cap);
  g.w2 = reinterpret_cast<const void* const*>(tl->fields + DWDP_TL_DOWN_WEIGHT_PTRS * cap);
  const bool scaled = tl->weight_dtype == DWDP_DTYPE_FP8_E4M3;
  g.s13 = scaled ? reinterpret_cast<const float* const*>(tl->fields + DWDP_TL_QUANTIZATION_PTRS * cap) : nullptr;
  g.s2 = scaled ? reinterpret_cast<const float* const*>(tl->fields + DWDP_TL_DOWN_QUANTIZATION_PTRS * cap) : nullptr;
  return moe_experts_checked(&g, shared, nullptr, packed_token_indices, hidden, num_tokens, top_k,
                             tl->fields + DWDP_TL_TOKEN_COUNTS * cap, tl->fields + DWDP_TL_TOKEN_OFFSETS * cap,
                             packed_weights, shared_gate, weighted_out, shared_out, workspace, workspace_bytes,
                             status, stream);
}

// --------------------------------------------------------------------------- decode-step attention pieces
extern "C" int dwdp_add_rmsnorm(void* residual, const void* delta, const void* weight, int64_t rows,
                                int hidden_size, float eps, void* out, void* stream) {
  g_last_error.clear();
  if (rows < 0 || hidden_size <= 0 || hidden_size % 8)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "add_rmsnorm: hidden_size must be a positive multiple of 8");
  if (rows > 0 && (residual == nullptr || weight == nullptr || out == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "add_rmsnorm: null pointer");
  return check(dwdp_add_rmsnorm_launch(residual, delta, weight, rows, hidden_size, eps, out, as_stream(stream)),
               "add_rmsnorm");
}

extern "C" int dwdp_rope_append_kv(const void* qkv, const void* qkv_bias, const int32_t* positions,
                                   const int32_t* block_table, int batch, int max_blocks, int num_blocks,
                                   int num_heads, int head_dim, int block_size, float rope_theta, void* q_out,
                                   void* k_cache, void* v_cache, int* status, void* stream) {
  g_last_error.clear();
  if (batch < 0 || num_heads <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 1024 || block_size <= 0 ||
      max_blocks <= 0 || num_blocks <= 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "rope_append_kv: bad sizes");
  if (batch > 0 && (qkv == nullptr || positions == nullptr || block_table == nullptr || q_out == nullptr ||
                    k_cache == nullptr || v_cache == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "rope_append_kv: null pointer");
  return check(dwdp_rope_append_launch(qkv, qkv_bias, positions, block_table, batch, max_blocks, num_blocks,
                                       num_heads, head_dim,
                                       block_size, rope_theta, q_out, k_cache, v_cache, status, as_stream(stream)),
               "rope_append_kv");
}

extern "C" size_t dwdp_paged_attention_workspace_bytes(int batch, int num_heads, int splits) {
  if (batch <= 0 || num_heads <= 0 || splits <= 0) return 0;
  return dwdp_paged_attention_workspace_bytes_impl(batch, num_heads, splits);
}

extern "C" int dwdp_paged_attention(const void* q, const void* k_cache, const void* v_cache,
                                    const int32_t* block_table, const int32_t* seq_lens, int batch, int max_blocks,
                                    int num_blocks, int num_heads, int head_dim, int block_size, int max_len,
                                    int splits, float scale, void* workspace, void* out, int* status, void* stream) {
  g_last_error.clear();
  if (batch < 0 || num_heads <= 0 || block_size <= 0 || max_blocks <= 0 || num_blocks <= 0 || splits <= 0 ||
      max_len <= 0 || max_len > max_blocks * block_size)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "paged_attention: bad sizes");
  if (head_dim != 128) return fail(DWDP_ERR_UNSUPPORTED, "paged_attention: head_dim must be 128");
  if (batch > 0 && (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_table == nullptr ||
                    seq_lens == nullptr || workspace == nullptr || out == nullptr))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "paged_attention: null pointer");
  return check(dwdp_paged_attention_launch(q, k_cache, v_cache, block_table, seq_lens, batch, max_blocks, num_blocks,
                                           num_heads,
                                           head_dim, block_size, max_len, splits, scale, workspace, out,
                                           status, as_stream(stream)),
               "paged_attention");
}

// --------------------------------------------------------------------------- expert-parallel decode exchange
extern "C" int dwdp_ep_dispatch(const void* hidden, const int64_t* topk_idx, const float* topk_weights,
                                int num_tokens, int top_k, int num_experts, int world, int rank, int hidden_size,
                                int capacity, const unsigned long long* peers, int* status, void* stream) {
  g_last_error.clear();
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_dispatch: world must be in [1, 8] and rank in [0, world)");
  if (num_tokens < 0 || top_k <= 0 || num_tokens * top_k > 2048 || num_tokens * top_k > capacity)
    return fail(DWDP_ERR_CAPACITY, "ep_dispatch: num_tokens * top_k must be <= min(2048, capacity)");
  if (hidden_size <= 0 || hidden_size % 8 || num_experts <= 0)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_dispatch: bad hidden_size / num_experts");
  if (peers == nullptr || (num_tokens > 0 && (hidden == nullptr || topk_idx == nullptr || topk_weights == nullptr)))
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_dispatch: null pointer");
  return check(dwdp_ep_dispatch_launch(hidden, topk_idx, topk_weights, num_tokens, top_k, num_experts, world, rank,
                                       hidden_size, capacity, peers, status, as_stream(stream)),
               "ep_dispatch");
}

extern "C" int dwdp_ep_plan(void* ep_buffer, int world, int rank, int hidden_size, int capacity, int num_experts,
                            int expert_lo, int local_experts, int64_t* counts, int64_t* offsets, int* packed_src,
                            float* packed_weights, int* ret_addr, int* total, void* packed_hidden, int* status,
                            void* stream) {
  g_last_error.clear();
  if (world < 1 || world > 8 || rank < 0 || rank >= world || local_experts <= 0 || local_experts > 256)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_plan: world in [1, 8], local_experts in [1, 256]");
  if (ep_buffer == nullptr || counts == nullptr || offsets == nullptr || packed_src == nullptr ||
      packed_weights == nullptr || ret_addr == nullptr || total == nullptr || packed_hidden == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_plan: null pointer");
  return check(dwdp_ep_plan_launch(ep_buffer, world, rank, hidden_size, capacity, num_experts, expert_lo,
                                   local_experts, counts, offsets, packed_src, packed_weights, ret_addr, total,
                                   packed_hidden, status, as_stream(stream)),
               "ep_plan");
}

extern "C" int dwdp_ep_combine(void* ep_buffer, int world, int rank, int hidden_size, int capacity,
                               const void* weighted, const int* ret_addr, const int* total,
                               const unsigned long long* peers, int* status, void* stream) {
  g_last_error.clear();
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_combine: world must be in [1, 8] and rank in [0, world)");
  if (ep_buffer == nullptr || weighted == nullptr || ret_addr == nullptr || total == nullptr || peers == nullptr)
    return fail(DWDP_ERR_INVALID_ARGUMENT, "ep_combine: null pointer");
  return check(dwdp_ep_combine_launch(ep_buffer, world, rank, hidden_size, capacity, weighted, ret_addr, total,
                                      peers, status, as_stream(stream)),
               "ep_combine");
}

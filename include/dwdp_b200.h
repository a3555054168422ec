/*
 * dwdp_b200.h — C ABI of the B200-native DWDP MoE-layer hot path.
 *
 * Plain C: raw device pointers, sizes, dtype codes and an opaque CUDA stream
 * (`void*` holding a cudaStream_t; NULL = legacy default stream). Every entry
 * point returns an int status (DWDP_OK = 0, negative on error) and never
 * throws; dwdp_last_error() returns a thread-local message for the last
 * failure on the calling thread.
 *
 * Reference interfaces each group replaces (paths inside the DWDP project):
 *   router    DWDP/router/kernels/fused.py:8-42 reference_topk_routing,
 *             DWDP/router/linear.py:38-44 compute_router_logits
 *   dispatch  DWDP/dispatcher/kernels/reference.py:163-257
 *             counting_scatter_expert_major_dispatch (+ ops/scatter.py:6-96)
 *   schedule  DWDP/scheduler/ops/round_robin.py:8-80 build_round_robin_schedule
 *   experts   DWDP/executor/pytorch.py:32-224 PyTorchExecutor.forward,
 *             DWDP/executor/kernels/persistent.py:160-226 / fp8.py:82-143,
 *             DWDP/executor/tensor_list.py:29-67 (pointer-array expert handles)
 *   weights   DWDP/executor/fp8.py:17-51, 118-146 (one-shot FP8 conversion)
 *   merge     DWDP/merger/kernels/reference.py:6-27 reference_merge
 *   shared    DWDP/adapters/qwen15_moe.py:302-319 _add_shared_expert
 */
#ifndef DWDP_B200_H_
#define DWDP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define DWDP_OK 0
#define DWDP_ERR_INVALID_ARGUMENT (-1)
#define DWDP_ERR_CAPACITY (-2)
#define DWDP_ERR_CUDA (-3)
#define DWDP_ERR_DEVICE_TIMEOUT (-4)
#define DWDP_ERR_DEVICE_BOUNDS (-5)
#define DWDP_ERR_UNSUPPORTED (-6)
#define DWDP_ERR_STATE (-7)
#define DWDP_ERR_NOT_FOUND (-8)

/* ---- dtype codes (1..3 follow DWDP/executor/tensor_list.py:237-246) ---- */
#define DWDP_DTYPE_F16 1
#define DWDP_DTYPE_BF16 2
#define DWDP_DTYPE_FP8_E4M3 3
#define DWDP_DTYPE_F32 4

/* ---- weight scale modes ------------------------------------------------ */
#define DWDP_SCALE_NONE 0     /* bf16 weights, no scale                     */
#define DWDP_SCALE_CHANNEL 1  /* fp8, one fp32 scale per output row         */
#define DWDP_SCALE_BLOCK128 2 /* fp8, one fp32 scale per 128x128 block      */
#define DWDP_SCALE_TENSOR 3   /* fp8, one fp32 scale per expert matrix
                                 (convert_qwen_weights_to_fp8_once with a
                                 scale_map, DWDP/executor/fp8.py:45-49);
                                 stored per row like CHANNEL, every row of a
                                 matrix holding the same value              */

/* ---- activation quantisation of the e4m3 expert GEMMs ------------------ */
#define DWDP_ACT_HILO 0     /* two e4m3 planes per row, v ~ s * (hi + lo/16),
                               one fp32 scale per row: about bf16 precision  */
#define DWDP_ACT_BLOCK128 1 /* one e4m3 plane, one fp32 scale per (row, 128
                               channels) = max(amax, 1e-5) / 448: the
                               reference's FP8 activation scheme
                               (DWDP/executor/fp8.py:86-115); the SwiGLU
                               intermediate is re-quantised the same way
                               (DWDP/executor/triton_tma.py:194-203)         */

/* Device status word: int[4] {code, where, detail, count} in device memory,
 * zeroed by the caller. Kernels record bounded-wait timeouts and failed bounds
 * checks there instead of trapping. May be NULL. */

int dwdp_version(void);
const char* dwdp_last_error(void);
/* Number of SMs of the current device (the persistent grid size). */
int dwdp_device_sm_count(void);

/* ======================================================================== *
 * Router: logits = x . W^T (+bias) (*score_scale) in fp32; top-k over logits
 * (ties -> lower expert id, slots in descending logit order); softmax over the
 * k selected; optional renormalisation by sum.clamp_min(eps); k == 1 gives
 * weight 1. renormalize == 2 instead gives each selected expert its probability
 * under the softmax over all E logits, not renormalised (the Hugging Face
 * Qwen2-MoE router with norm_topk_prob = false). Optionally the sigmoid
 * shared-expert gate sigmoid(x . g).
 * Replaces reference_topk_routing + compute_router_logits (fused.py:8-42,
 * linear.py:38-44). E <= 256, K <= 16.
 *   hidden [T,H] (hidden_dtype bf16|f32), weight [E,H] (weight_dtype bf16|f32)
 *   bias [E] f32 or NULL, shared_gate_weight [H] (weight_dtype) or NULL
 *   logits [T,E] f32 (required), probs [T,K] f32 (may be NULL), topk_weights [T,K] f32,
 *   topk_idx [T,K] int64, shared_gate [T] f32 (NULL when no gate weight)
 * ======================================================================== */
int dwdp_router_topk(const void* hidden, int hidden_dtype, const void* weight, int weight_dtype,
                     const float* bias, const void* shared_gate_weight, int64_t num_tokens,
                     int hidden_size, int num_experts, int top_k, float score_scale,
                     int renormalize, float eps, float* logits, float* probs, int64_t* topk_idx,
                     float* topk_weights, float* shared_gate, int* status, void* stream);

/* ======================================================================== *
 * Dispatch: stable counting sort of the T*K token-major assignments into
 * expert-major order, bit-exact with counting_scatter_expert_major_dispatch
 * (reference.py:163-257): dest[i] = offsets[e_i] + #{j < i : e_j == e_i}.
 *   counts [E], offsets [E+1], perm/inv/ids/tok [T*K]  (all int64)
 *   packed_weights [T*K] in weight_dtype (f32|bf16|f16), bit-copied
 *   hidden/packed_hidden: optional bf16 row gather packed_hidden[d] = hidden[tok[d]]
 *   (hidden_size columns); pass NULL to skip.
 *   scratch: dwdp_dispatch_scratch_bytes() bytes of device memory.
 * ======================================================================== */
size_t dwdp_dispatch_scratch_bytes(int64_t num_tokens, int top_k, int num_experts);
int dwdp_dispatch(const int64_t* topk_idx, const void* topk_weights, int weight_dtype,
                  int64_t num_tokens, int top_k, int num_experts, int64_t* counts,
                  int64_t* offsets, int64_t* perm, int64_t* inv, int64_t* ids, int64_t* tok,
                  void* packed_weights, const void* hidden, int hidden_size, void* packed_hidden,
                  void* scratch, int* status, void* stream);

/* Row gather alone (the executor's input gather, executor/ops gather_expert_inputs):
 * packed[d] = hidden[token_index[d]] for d < num_rows, bf16 rows of hidden_size. */
int dwdp_gather_rows(const void* hidden, const int64_t* token_index, int64_t num_rows, int hidden_size,
                     int64_t num_tokens, void* packed, int* status, void* stream);

/* Allocation-free variant of dwdp_dispatch (no counterpart in the reference).
 * For callers that cannot allocate device memory at dispatch time: a serving
 * loop under a fixed memory budget, a plugin that only sees one call's tensors,
 * a host with no device allocator. Same arguments and results as dwdp_dispatch
 * minus `scratch`: the histogram scratch is a fixed 1 MiB array inside the
 * library (held by every GPU that loads it until exit), so
 * ceil(T*K/256) * E must be <= 262144 or DWDP_ERR_CAPACITY is returned. The
 * first call on a device looks the array up (cudaGetSymbolAddress) and should
 * come before any stream capture; calls that overlap on the GPU share the array
 * and race. It allocates nothing. */
int dwdp_dispatch_noalloc(const int64_t* topk_idx, const void* topk_weights, int weight_dtype,
                          int64_t num_tokens, int top_k, int num_experts, int64_t* counts,
                          int64_t* offsets, int64_t* perm, int64_t* inv, int64_t* ids, int64_t* tok,
                          void* packed_weights, const void* hidden, int hidden_size,
                          void* packed_hidden, int* status, void* stream);
size_t dwdp_dispatch_noalloc_max_scratch_bytes(void);

/* ======================================================================== *
 * Activation quantisation alone (quantize_activations_blockwise,
 * DWDP/executor/fp8.py:86-115): one e4m3 plane with one fp32 scale per
 * (row, 128 channels), scale = max(amax, 1e-5) / 448, q = e4m3(v / scale)
 * (IEEE division, round to nearest even): bytes and scales equal the
 * reference's. The grouped GEMMs run the same quantiser in their planning
 * launch (DWDP_ACT_BLOCK128).
 *   src bf16 [src_rows, cols]; row r of the output reads src row row_index[r]
 *   (int64, NULL = row r; an out-of-range index quantises a zero row and sets
 *   DWDP_ERR_DEVICE_BOUNDS in *status). cols % 128 == 0.
 *   dst e4m3 [rows, cols]; scales fp32 [rows][cols/128] (scale_layout 0, the
 *   reference's layout) or [cols/128][rows] (scale_layout 1).
 * ======================================================================== */
int dwdp_quantize_activations_blockwise(const void* src, int64_t src_rows, const int64_t* row_index,
                                        int64_t rows, int cols, void* dst, float* scales, int scale_layout,
                                        int* status, void* stream);

/* ======================================================================== *
 * Router + dispatch in ONE launch for decode-sized batches: dwdp_router_topk
 * followed by dwdp_dispatch (fp32 routing weights, no row gather) with the same
 * outputs and meaning, for bf16 hidden and weights, 0 < T * K <= 256, E <= 256,
 * K <= 16. One CTA per expert row (and one for the shared gate) computes that
 * row's logits for every token; the last CTA to finish routes every token and
 * sorts the T * K assignments (the reference counting scatter,
 * DWDP/dispatcher/kernels/reference.py:163-257, after DWDP/router/kernels/fused.py:8-42).
 *   gate_logit [T] f32 scratch (needed with a shared gate weight);
 *   ticket: one int32 of device memory, zero before the first call; the kernel
 *   returns it to zero, so a stream's consecutive calls may share it (calls that
 *   overlap on the GPU must not).
 * Outside that range: DWDP_ERR_UNSUPPORTED (use the two stages).
 * ======================================================================== */
int dwdp_route_dispatch_small(const void* hidden, const void* weight, const float* bias,
                              const void* shared_gate_weight, int64_t num_tokens, int hidden_size, int num_experts,
                              int top_k, float score_scale, int renormalize, float eps, float* logits,
                              float* gate_logit, float* probs, int64_t* topk_idx, float* topk_weights,
                              float* shared_gate, int64_t* counts, int64_t* offsets, int64_t* perm, int64_t* inv,
                              int64_t* ids, int64_t* tok, float* packed_weights, int* ticket, int* status,
                              void* stream);

/* ======================================================================== *
 * Round-robin schedule over active experts in ascending id
 * (build_round_robin_schedule, round_robin.py:8-80), padded to E entries:
 * rows [0, num_active) hold the reference values, the rest are -1.
 *   out arrays [E] int64: expert_queue, starts, ends, active_counts,
 *   priority (= order), stream_ids (= order % stream_count); num_active [1].
 * ======================================================================== */
int dwdp_schedule(const int64_t* counts, const int64_t* offsets, int num_experts,
                  int stream_count, int64_t* expert_queue, int64_t* starts, int64_t* ends,
                  int64_t* active_counts, int64_t* priority, int64_t* stream_ids,
                  int64_t* num_active, void* stream);

/* ======================================================================== *
 * Expert weight store. Weights are kept pre-tiled in the layout the grouped
 * GEMM streams: for an [R, Kd] projection (R output rows, Kd inputs, both
 * multiples of 128) tiles of 128 rows x TK inputs, tile (rb, kb) of matrix p
 * of a P-matrix pack at tile index (rb * (Kd/TK) + kb) * P + p.
 *   FP8 (every scale mode): TK = 128, 16384-byte tiles of 128-byte rows in
 *                 the 128-byte-swizzled smem image (chunk c of row r at
 *                 c ^ (r&7)); scales fp32 [P][R] (CHANNEL, TENSOR) or
 *                 [P][R/128][Kd/128] (BLOCK128).
 *   BF16        : TK = 64, 16384-byte tiles in the 128-byte-swizzled image.
 * Quantisation follows DWDP/executor/fp8.py:118-146: scale = max(amax, 1e-5)
 * / 448, q = e4m3(w / scale) (round to nearest even, IEEE division).
 * Gate/up are packed together (P = 2, gate then up) so one tile fetch brings
 * both halves of a SwiGLU feature block.
 *   src_mats: host array of P device pointers to row-major [R, Kd] matrices
 *   (src_dtype bf16|f32).
 * ======================================================================== */
size_t dwdp_packed_weight_bytes(int rows, int cols, int num_mats, int dst_dtype);
size_t dwdp_packed_scale_floats(int rows, int cols, int num_mats, int scale_mode);
int dwdp_pack_weights(const void* const* src_mats, int src_dtype, int rows, int cols,
                      int num_mats, int dst_dtype, int scale_mode, void* dst_tiles,
                      float* dst_scales, void* stream);
/* Inverse of dwdp_pack_weights: dequantised fp32 [P][R][Kd]. */
int dwdp_unpack_weights(const void* tiles, const float* scales, int rows, int cols,
                        int num_mats, int dst_dtype, int scale_mode, float* out,
                        void* stream);

/* ======================================================================== *
 * Expert group: the device-resident handle set one grouped GEMM launch reads
 * (the TensorList pointer arrays of tensor_list.py:29-67, reduced to what the
 * kernel needs). Pointer arrays live in device memory, one entry per expert.
 * ======================================================================== */
typedef struct dwdp_expert_group {
  int num_experts;
  int hidden_size;         /* H: K of gate/up, output width of down       */
  int intermediate_size;   /* I: output width of gate/up, K of down       */
  int weight_dtype;        /* DWDP_DTYPE_BF16 | DWDP_DTYPE_FP8_E4M3       */
  int scale_mode;          /* DWDP_SCALE_*                                */
  const void* const* w13;  /* [E] packed gate/up tiles (num_mats = 2)     */
  const void* const* w2;   /* [E] packed down tiles (num_mats = 1)        */
  const float* const* s13; /* [E] gate/up scales                          */
  const float* const* s2;  /* [E] down scales                             */
  int act_quant;           /* DWDP_ACT_* (e4m3 weights only; a shared group
                              follows the routed group's setting)          */
} dwdp_expert_group;

/* ======================================================================== *
 * Grouped expert execution (replaces PyTorchExecutor.forward's per-expert
 * loop, pytorch.py:66-160): for every routed assignment row d
 *   weighted_out[d] = w[d] * down(silu(gate(xd)) * up(xd)),  xd = packed_hidden[d]
 * and, when `shared` is given, for every token t
 *   sum_p shared_out[p][t] = shared_gate[t] * down_s(silu(gate_s(x_t)) * up_s(x_t))
 * (shared_gate NULL = 1; p < dwdp_moe_shared_parts(T, Is), shared_out is
 * [parts][T][H] bf16). bf16 activations, fp32 accumulation in TMEM,
 * bf16 outputs. Two persistent tcgen05 GEMM launches (gate/up+SwiGLU,
 * down+scale) after a planning launch. Per-channel fp8 weights run as e4m3
 * MMAs (kind::f8f6f4) against activations carried as two e4m3 planes
 * (hi + lo/16, one fp32 scale per row, about bf16 precision), quantised in the
 * planning launch and in one launch between the GEMMs; block-scaled fp8 and
 * bf16 weights run as bf16 MMAs. Expert row ranges come from device offsets;
 * no host synchronisation. hidden_size <= 8192. The shared group must use the
 * routed group's weight dtype and scale mode.
 * ======================================================================== */
/* Number of [T, H] partial slabs `shared_out` must hold: the shared expert's
 * down projection is split along K at decode sizes (its K is several times the
 * routed one) and the merge sums the partials. */
int dwdp_moe_shared_parts(int64_t num_tokens, int shared_intermediate_size);
size_t dwdp_moe_workspace_bytes(int64_t num_tokens, int top_k, int num_experts,
                                int intermediate_size, int shared_intermediate_size);
int dwdp_moe_experts(const dwdp_expert_group* routed, const dwdp_expert_group* shared,
                     const void* packed_hidden, const void* hidden, int64_t num_tokens,
                     int top_k, const int64_t* counts, const int64_t* offsets,
                     const float* packed_weights, const float* shared_gate, void* weighted_out,
                     void* shared_out, void* workspace, size_t workspace_bytes, int* status,
                     void* stream);

/* As dwdp_moe_experts, with routed row d read as hidden[packed_token_indices[d]]
 * (the dispatcher's packed_token_indices) instead of from a gathered
 * packed_hidden: the e4m3 path quantises straight from `hidden`, so the
 * dispatcher's row gather can be skipped. */
int dwdp_moe_experts_indexed(const dwdp_expert_group* routed, const dwdp_expert_group* shared,
                             const int64_t* packed_token_indices, const void* hidden, int64_t num_tokens,
                             int top_k, const int64_t* counts, const int64_t* offsets,
                             const float* packed_weights, const float* shared_gate, void* weighted_out,
                             void* shared_out, void* workspace, size_t workspace_bytes, int* status,
                             void* stream);

/* The shared expert alone: for every token t, sum_p shared_out[p][t] =
 * g_t * down_s(silu(gate_s(x_t)) * up_s(x_t)), p < dwdp_moe_shared_parts(T, Is).
 * shared_gate == NULL: g_t = 1 (ungated; dwdp_merge_gated applies the gate later),
 * so it depends only on `hidden` and can start before the router. With the router's
 * shared_gate [T] the gate is applied in the down epilogue exactly as
 * dwdp_moe_experts does for its shared rows (bit-identical partials). */
size_t dwdp_moe_shared_workspace_bytes(int64_t num_tokens, int hidden_size, int shared_intermediate_size);
int dwdp_moe_shared_expert(const dwdp_expert_group* shared, const void* hidden, int64_t num_tokens,
                           const float* shared_gate, void* shared_out, void* workspace, size_t workspace_bytes,
                           int* status, void* stream);

/* ======================================================================== *
 * TensorList (DWDP/executor/tensor_list.py:29-228): the non-owning
 * structure-of-arrays descriptor of the active experts. `fields` is one device
 * int64 buffer of DWDP_TL_ROWS rows x `capacity` entries; rows 0..25 are the
 * reference's fields in its order (tensor_list.py:201-228), row 26 holds the
 * down-projection scale address (the reference has one quantization_ptrs row,
 * left 0, tensor_list.py:160; here quantization_ptrs is the gate/up scale
 * address). Entries past the active count are empty (count 0, null pointers,
 * expert id -1), so a launch over all `capacity` entries needs no host count.
 * gate_weight_ptrs and up_weight_ptrs name the same packed gate/up slab.
 * ======================================================================== */
#define DWDP_TL_INPUT_PTRS 0
#define DWDP_TL_TOKEN_INDEX_PTRS 1
#define DWDP_TL_ROUTING_WEIGHT_PTRS 2
#define DWDP_TL_GATE_WEIGHT_PTRS 3
#define DWDP_TL_UP_WEIGHT_PTRS 4
#define DWDP_TL_DOWN_WEIGHT_PTRS 5
#define DWDP_TL_INTERMEDIATE_PTRS 6
#define DWDP_TL_OUTPUT_PTRS 7
#define DWDP_TL_WEIGHTED_OUTPUT_PTRS 8
#define DWDP_TL_QUANTIZATION_PTRS 9
#define DWDP_TL_EXPERT_IDS 10
#define DWDP_TL_TOKEN_OFFSETS 11
#define DWDP_TL_TOKEN_COUNTS 12
#define DWDP_TL_M 13
#define DWDP_TL_N 14
#define DWDP_TL_K 15
#define DWDP_TL_INTERMEDIATE_N 16
#define DWDP_TL_INPUT_LD 17
#define DWDP_TL_GATE_LD 18
#define DWDP_TL_UP_LD 19
#define DWDP_TL_DOWN_LD 20
#define DWDP_TL_OUTPUT_LD 21
#define DWDP_TL_DTYPE_CODES 22
#define DWDP_TL_WORKSPACE_INDICES 23
#define DWDP_TL_EXECUTION_PRIORITIES 24
#define DWDP_TL_STREAM_IDS 25
#define DWDP_TL_DOWN_QUANTIZATION_PTRS 26
#define DWDP_TL_ROWS 27

/* Storage the pointer fields describe (the same for every entry, row-offset by
 * the entry's token_offsets): what TensorList.from_plans reads off its tensors. */
typedef struct dwdp_tensor_list_bases {
  const void* input;            /* hidden_states [T, H]                       */
  const void* token_index;      /* packed_token_indices [N] int64             */
  const void* routing_weights;  /* packed_routing_weights [N]                 */
  const void* intermediate;     /* [N, intermediate_n] or NULL                */
  const void* output;           /* packed outputs [N, n] or NULL              */
  const void* weighted_output;  /* weighted outputs [N, n] or NULL            */
  int64_t intermediate_row_bytes, output_row_bytes, weighted_row_bytes;
  int64_t n, k, intermediate_n, input_ld, gate_ld, up_ld, down_ld, output_ld, dtype_code;
} dwdp_tensor_list_bases;

typedef struct dwdp_tensor_list {
  int64_t capacity;        /* entries per field row (<= 1024)                */
  int64_t* fields;         /* device [DWDP_TL_ROWS][capacity] int64          */
  int hidden_size, intermediate_size, weight_dtype, scale_mode, act_quant;
} dwdp_tensor_list;

/* Fill `tl->fields` from an execution plan (expert_queue / expert_starts /
 * expert_counts / execution_priority / stream_assignments of plan_len rows;
 * priorities and streams may be NULL) and the experts' pointer arrays
 * (TensorList.from_plans, tensor_list.py:69-198): rows with expert id >= 0 and
 * count > 0 are compacted in plan order. meta[0] = active entries, meta[1] =
 * the largest token count (device int64[2]). One launch, no host sync. Plan
 * rows beyond capacity: DWDP_ERR_CAPACITY in *status. */
int dwdp_tensor_list_build(const int64_t* expert_queue, const int64_t* expert_starts,
                           const int64_t* expert_counts, const int64_t* priorities, const int64_t* stream_ids,
                           int plan_len, const dwdp_expert_group* experts, const dwdp_tensor_list_bases* bases,
                           const dwdp_tensor_list* tl, int64_t* meta, int* status, void* stream);

/* The grouped expert GEMMs driven by a TensorList (the dwdp_grouped_moe entry
 * the reference's persistent Triton executors correspond to,
 * executor/kernels/persistent.py:160-226): every entry i with token_counts[i] > 0
 * computes weighted_out[r] = w[r] * down(silu(gate(x_r)) * up(x_r)) for its rows
 * r in [token_offsets[i], token_offsets[i] + token_counts[i]), x_r =
 * hidden[packed_token_indices[r]], reading its weights from the entry's pointer
 * fields. `shared` and the rest as dwdp_moe_experts_indexed; the workspace is
 * dwdp_moe_workspace_bytes(num_tokens, top_k, tl->capacity, I, Is). */
int dwdp_grouped_moe(const dwdp_tensor_list* tl, const dwdp_expert_group* shared,
                     const int64_t* packed_token_indices, const void* hidden, int64_t num_tokens, int top_k,
                     const float* packed_weights, const float* shared_gate, void* weighted_out,
                     void* shared_out, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* ======================================================================== *
 * Merge (reference_merge, merger/kernels/reference.py:6-27): deterministic
 * token-major reduction. out[t] = sum over the K rows inv[t*K+k] of
 * weighted[row] taken in ascending row order, plus shared_out[p][t] for
 * p < shared_parts (<= 8) when shared_out is given. fp32 accumulation; out_dtype
 * bf16|f32; weighted/shared bf16. K <= 16.
 * ======================================================================== */
int dwdp_merge(const void* weighted, const int64_t* inv, const void* shared_out, int shared_parts,
               int64_t num_tokens, int top_k, int hidden_size, void* out, int out_dtype,
               void* stream);
/* As dwdp_merge with ungated shared partials: out[t] = routed sum + shared_gate[t] *
 * (sum over the shared parts), the gate applied in fp32 (DWDP/adapters/qwen15_moe.py:302-319). */
int dwdp_merge_gated(const void* weighted, const int64_t* inv, const void* shared_out, int shared_parts,
                     const float* shared_gate, int64_t num_tokens, int top_k, int hidden_size, void* out,
                     int out_dtype, void* stream);

/* ======================================================================== *
 * Decode-step attention pieces (the model around the MoE layers for a full
 * Qwen1.5-MoE decode step; DWDP/adapters/qwen15_moe.py:526-543 captures the HF
 * decoder layers around the DWDP blocks). bf16 tensors, fp32 arithmetic.
 * The paged KV cache follows DWDP/runtime/paged_attention.py:20-76: per layer a
 * K and a V array [num_blocks, block_size, num_heads, head_dim]; sequence b's
 * position p lives in block block_table[b * max_blocks + p / block_size] (int32).
 * ======================================================================== */
/* residual[r] += delta[r] (skipped when delta is NULL); out[r] = rmsnorm(residual[r]) * weight
 * (Qwen2RMSNorm: x * rsqrt(mean(x^2) + eps), fp32). hidden_size % 8 == 0. */
int dwdp_add_rmsnorm(void* residual, const void* delta, const void* weight, int64_t rows, int hidden_size,
                     float eps, void* out, void* stream);
/* qkv [batch, 3, num_heads, head_dim] (+ qkv_bias [3, num_heads, head_dim] when given):
 * q_out [batch, num_heads, head_dim] gets q with the rotary embedding at positions[b]
 * (NeoX rotate-half, inv_freq_d = rope_theta^(-2d/head_dim)); the rotated k and v are
 * written into the caches ([num_blocks, block_size, num_heads, head_dim]) at positions[b].
 * A position outside [0, max_blocks * block_size) or a block id outside [0, num_blocks):
 * DWDP_ERR_DEVICE_BOUNDS in *status, the token skipped (q_out and the caches untouched). */
int dwdp_rope_append_kv(const void* qkv, const void* qkv_bias, const int32_t* positions,
                        const int32_t* block_table, int batch, int max_blocks, int num_blocks, int num_heads,
                        int head_dim, int block_size, float rope_theta, void* q_out, void* k_cache, void* v_cache,
                        int* status, void* stream);
size_t dwdp_paged_attention_workspace_bytes(int batch, int num_heads, int splits);
/* out[b, h] = softmax(scale * q[b, h] . K[b, :seq_lens[b], h]) V[b, :seq_lens[b], h] for one
 * query per sequence. The context is split into `splits` chunks of ceil(max_len / splits)
 * positions per (sequence, head), combined with the log-sum-exp rescaling. head_dim 128;
 * max_len >= every seq_lens[b] and <= max_blocks * block_size. A block id outside
 * [0, num_blocks) (its positions are skipped) or a pipeline wait that runs out:
 * DWDP_ERR_DEVICE_BOUNDS / _TIMEOUT in *status (may be NULL). */
int dwdp_paged_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                         const int32_t* seq_lens, int batch, int max_blocks, int num_blocks, int num_heads,
                         int head_dim, int block_size, int max_len, int splits, float scale, void* workspace,
                         void* out, int* status, void* stream);

/* ======================================================================== *
 * Expert-parallel decode exchange (replaces the all_to_all_single EP path of
 * DWDP/adapters/qwen15_moe.py:164-243, used below ep_batch_size_threshold,
 * DWDP/runtime/config.py:31). Every rank allocates one EP buffer of
 * dwdp_ep_buffer_bytes(world, H, capacity) bytes (capacity = T_max * top_k rows), exports
 * it with dwdp_export_ipc_handle and opens the others' with dwdp_ipc_open; `peers` is a
 * DEVICE array of world base addresses (this rank's own buffer at [rank]). Expert e is
 * owned by rank min(e / ceil(E / world), world - 1). All ranks use the same top_k and
 * capacity; each rank's num_tokens may differ (0 <= num_tokens * top_k <= capacity), and
 * a rank with no tokens still runs every step (the owners count one arrival per send CTA
 * of every source). Per forward, in stream order:
 *   dwdp_ep_dispatch   rows of every (token, slot) -> the owner's buffer;
 *   dwdp_ep_plan       owner: wait for every rank, counting sort by local expert into
 *                      counts/offsets (local_experts entries, int64), packed_src, packed
 *                      routing weights, return addresses, *total, and the packed rows;
 *   (grouped GEMMs over the received rows: dwdp_moe_experts with packed_hidden sized
 *    for world * capacity rows, num_tokens = world * capacity and top_k = 1)
 *   dwdp_ep_combine    weighted rows back to their source's buffer, then wait for all
 *                      owners; the source's results are then the rows
 *                      [dwdp_ep_ret_offset(), + num_tokens * top_k * H * 2) of its own
 *                      buffer in slot order (merge them with an identity inverse).
 * Waits are bounded (about a second): DWDP_ERR_DEVICE_TIMEOUT in *status.
 * ======================================================================== */
size_t dwdp_ep_buffer_bytes(int world, int hidden_size, int capacity);
size_t dwdp_ep_ret_offset(int world, int hidden_size, int capacity);
int dwdp_ipc_open(const void* handle, size_t offset, void** base_out, void** ptr_out);
int dwdp_ipc_close(void* base);
int dwdp_ep_dispatch(const void* hidden, const int64_t* topk_idx, const float* topk_weights, int num_tokens,
                     int top_k, int num_experts, int world, int rank, int hidden_size, int capacity,
                     const unsigned long long* peers, int* status, void* stream);
int dwdp_ep_plan(void* ep_buffer, int world, int rank, int hidden_size, int capacity, int num_experts,
                 int expert_lo, int local_experts, int64_t* counts, int64_t* offsets, int* packed_src,
                 float* packed_weights, int* ret_addr, int* total, void* packed_hidden, int* status,
                 void* stream);
int dwdp_ep_combine(void* ep_buffer, int world, int rank, int hidden_size, int capacity, const void* weighted,
                    const int* ret_addr, const int* total, const unsigned long long* peers, int* status,
                    void* stream);

/* ======================================================================== *
 * DWDP communication engine (replaces the pybind module dwdp_communication_ext,
 * DWDP/communication/bindings.cpp:32-111): expert slabs sharded across the GPUs
 * of one box, remote slabs opened through CUDA IPC (or a peer pointer) and
 * copied by the copy engines into `num_buffers` staging buffers of `num_slots`
 * fixed slots on a greatest-priority stream; prefetch/wait per buffer, the wait
 * ordered on the caller's stream. Messages: dwdp_engine_last_error().
 * ======================================================================== */
typedef struct dwdp_engine dwdp_engine;
const char* dwdp_engine_last_error(void);
size_t dwdp_ipc_handle_bytes(void);
/* export_ipc_handle (bindings.cpp:27-30): handle of the allocation holding ptr
 * plus ptr's byte offset inside it. */
int dwdp_export_ipc_handle(const void* device_ptr, void* handle_out, size_t* offset_out);
/* PeerTopology.canAccess (topology.cpp:17-41) */
int dwdp_peer_can_access(int src_device, int dst_device, int* out);
int dwdp_engine_create(int device_id, size_t slot_bytes, int num_slots, int num_buffers,
                       dwdp_engine** out);
int dwdp_engine_destroy(dwdp_engine* engine);
int dwdp_engine_register_local(dwdp_engine* engine, int expert_id, const void* ptr, size_t bytes);
int dwdp_engine_register_ipc(dwdp_engine* engine, int expert_id, const void* handle, size_t offset,
                             size_t bytes, int owner_device);
int dwdp_engine_register_peer(dwdp_engine* engine, int expert_id, const void* peer_ptr,
                              size_t bytes, int owner_device);
/* Copy the listed remote experts into `buffer` (local ones are skipped); when
 * after_stream is given the copies start after the work already queued on it. */
int dwdp_engine_prefetch(dwdp_engine* engine, const int* expert_ids, int n, int buffer,
                         void* after_stream);
/* One planned copy of a communication plan (the reference's CommunicationDescriptor,
 * DWDP/comms_planner/metadata.py:12-26): bytes [start, start + bytes) of the expert's
 * slab into the same offsets of its staging slot. */
typedef struct dwdp_copy_slice {
  int expert_id;
  int reserved;
  uint64_t start;
  uint64_t bytes;
} dwdp_copy_slice;
/* Execute a plan's descriptors into `buffer` in the given order (the reference's sliced
 * copyToNextAsync, communication/buffers.cu:94-134, with the slice order the planner and
 * the TransferScheduler chose): copy k runs on copy stream k % streams, or all of them in
 * SM copy kernels in DWDP_COPY_SM mode; slices of local experts are skipped; one event
 * marks the buffer ready for dwdp_engine_wait. A slice beyond its expert's bytes:
 * DWDP_ERR_INVALID_ARGUMENT, an unregistered expert: DWDP_ERR_NOT_FOUND (nothing issued). */
int dwdp_engine_prefetch_slices(dwdp_engine* engine, const dwdp_copy_slice* slices, int n, int buffer,
                                void* after_stream);
int dwdp_engine_wait(dwdp_engine* engine, int buffer, void* stream);
int dwdp_engine_resident_pointer(dwdp_engine* engine, int expert_id, int buffer, void** out);
int dwdp_engine_is_remote(dwdp_engine* engine, int expert_id, int* out);
int dwdp_engine_release(dwdp_engine* engine, int expert_id);
int dwdp_engine_synchronize(dwdp_engine* engine);
int dwdp_engine_stats(dwdp_engine* engine, unsigned long long* bytes_copied,
                      unsigned long long* copies_issued, void** copy_stream);

/* Copy mechanism of dwdp_engine_prefetch: DWDP_COPY_ENGINE (default) issues one
 * cudaMemcpyAsync per expert (or per slice) on the engine's copy streams, as the
 * reference's buffers.cu did; DWDP_COPY_SM launches dwdp_peer_copy_sm with `ctas`
 * CTAs on copy stream 0 (SMs load the peer's slab and store it locally). */
#define DWDP_COPY_ENGINE 0
#define DWDP_COPY_SM 1
int dwdp_engine_set_copy_mode(dwdp_engine* engine, int mode, int ctas);

/* Up to DWDP_COPY_LIST_MAX copies for one dwdp_peer_copy_sm launch (passed by value
 * as a kernel parameter). Every pointer 16-byte aligned. */
#define DWDP_COPY_LIST_MAX 64
typedef struct dwdp_copy_list {
  int n;
  const void* src[DWDP_COPY_LIST_MAX];
  void* dst[DWDP_COPY_LIST_MAX];
  size_t bytes[DWDP_COPY_LIST_MAX];
} dwdp_copy_list;
int dwdp_peer_copy_sm(const dwdp_copy_list* list, int ctas, void* stream);

/* CommunicationPolicy.decide (communication_policy.cpp:5-17); CommunicationPath codes. */
#define DWDP_PATH_LOCAL 0
#define DWDP_PATH_P2P 1
#define DWDP_PATH_IPC 2
#define DWDP_PATH_COPY 3
#define DWDP_RESIDENT_NONE 0
#define DWDP_RESIDENT_STAGED 1
#define DWDP_RESIDENT_ACTIVE 2
int dwdp_policy_decide(int local_gpu, int owner_gpu, int resident_state, int has_ipc_handle,
                       int peer_access);

/* TransferScheduler (transfer_scheduler.cpp:15-104): priority queue with
 * coalescing, two retries, cancel-while-queued, bounded take(). */
#define DWDP_TRANSFER_CREATED 0
#define DWDP_TRANSFER_QUEUED 1
#define DWDP_TRANSFER_RUNNING 2
#define DWDP_TRANSFER_WAITING 3
#define DWDP_TRANSFER_COMPLETED 4
#define DWDP_TRANSFER_FAILED 5
#define DWDP_TRANSFER_CANCELLED 6
typedef struct dwdp_sched dwdp_sched;
int dwdp_sched_create(dwdp_sched** out);
int dwdp_sched_destroy(dwdp_sched* s);
int dwdp_sched_submit(dwdp_sched* s, int expert_id, int priority);
int dwdp_sched_take(dwdp_sched* s, int timeout_ms, int* expert_id);
int dwdp_sched_complete(dwdp_sched* s, int expert_id);
int dwdp_sched_fail(dwdp_sched* s, int expert_id, int retryable);
int dwdp_sched_cancel(dwdp_sched* s, int expert_id);
int dwdp_sched_close(dwdp_sched* s);
int dwdp_sched_state(dwdp_sched* s, int expert_id, int* state, int* retries);

#ifdef __cplusplus
}
#endif

#endif /* DWDP_B200_H_ */

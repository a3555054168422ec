"""Tensor-level wrappers over the C ABI: torch supplies device memory and the
current CUDA stream; every computation runs in the hand-written sm_100a kernels.

Each function validates like the reference op it replaces (``ValueError`` on a
contract violation) and raises ``RuntimeError`` when the extension is missing or
a tensor is not on a CUDA device. Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

_DTYPE_CODES = {
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float8_e4m3fn: _lib.DTYPE_FP8_E4M3,
    torch.float32: _lib.DTYPE_F32,
}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {dtype}") from exc


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("DWDP B200 ops need CUDA tensors; there is no CPU fallback")


# --------------------------------------------------------------------------- router
@dataclass
class RouterResult:
    router_logits: torch.Tensor  # [T, E] fp32
    routing_probabilities: torch.Tensor  # [T, K] fp32
    topk_indices: torch.Tensor  # [T, K] int64
    topk_weights: torch.Tensor  # [T, K] fp32
    shared_gate: torch.Tensor | None  # [T] fp32


def router_topk(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    top_k: int,
    *,
    bias: torch.Tensor | None = None,
    shared_gate_weight: torch.Tensor | None = None,
    score_scale: float = 1.0,
    renormalize: bool = True,
    eps: float = 1e-9,
    out: RouterResult | None = None,
) -> RouterResult:
    """Fused logits + top-k + softmax-over-k + renormalisation (fp32 math).

    Mirrors ``LinearTopKRouter.compute_router_logits`` + ``reference_topk_routing``
    (DWDP/router/linear.py:38-44, DWDP/router/kernels/fused.py:8-42). Slots come
    out in descending logit order; ties go to the lower expert id.
    """
    _require_cuda(hidden, weight, bias, shared_gate_weight)
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H).contiguous()
    T = x.shape[0]
    E = weight.shape[0]
    if weight.ndim != 2 or weight.shape[1] != H:
        raise ValueError("router weight must be [num_experts, hidden_size]")
    w = weight.contiguous()
    if shared_gate_weight is not None:
        shared_gate_weight = shared_gate_weight.reshape(-1).to(w.dtype).contiguous()
        if shared_gate_weight.numel() != H:
            raise ValueError("shared gate weight must have hidden_size elements")
    dev = x.device
    if out is None:
        out = RouterResult(
            router_logits=torch.empty(T, E, dtype=torch.float32, device=dev),
            routing_probabilities=torch.empty(T, top_k, dtype=torch.float32, device=dev),
            topk_indices=torch.empty(T, top_k, dtype=torch.int64, device=dev),
            topk_weights=torch.empty(T, top_k, dtype=torch.float32, device=dev),
            shared_gate=(torch.empty(T, dtype=torch.float32, device=dev)
                         if shared_gate_weight is not None else None),
        )
    if T == 0:  # nothing to route (empty tensors have no data pointer to pass)
        return out
    b = None if bias is None else bias.float().contiguous()
    rc = _lib.load().dwdp_router_topk(
        x.data_ptr(), dtype_code(x.dtype), w.data_ptr(), dtype_code(w.dtype), _ptr(b),
        _ptr(shared_gate_weight), T, H, E, top_k, float(score_scale), int(renormalize), float(eps),
        _ptr(out.router_logits), _ptr(out.routing_probabilities), _ptr(out.topk_indices),
        _ptr(out.topk_weights), _ptr(out.shared_gate), None, _stream(),
    )
    _lib.check(rc, "router_topk")
    return out


# --------------------------------------------------------------------------- dispatch
@dataclass
class DispatchResult:
    expert_counts: torch.Tensor  # [E] int64
    expert_offsets: torch.Tensor  # [E+1] int64
    token_permutation: torch.Tensor  # [N] int64
    inverse_permutation: torch.Tensor  # [N] int64
    packed_expert_ids: torch.Tensor  # [N] int64
    packed_token_indices: torch.Tensor  # [N] int64
    packed_routing_weights: torch.Tensor  # [N] weight dtype
    packed_hidden: torch.Tensor | None  # [N, H] bf16


def dispatch_scratch_bytes(num_tokens: int, top_k: int, num_experts: int) -> int:
    return int(_lib.load().dwdp_dispatch_scratch_bytes(num_tokens, top_k, num_experts))


def dispatch(
    topk_indices: torch.Tensor,
    topk_weights: torch.Tensor,
    num_experts: int,
    *,
    hidden: torch.Tensor | None = None,
    scratch: torch.Tensor | None = None,
    out: DispatchResult | None = None,
    status: torch.Tensor | None = None,
) -> DispatchResult:
    """Stable counting-sort dispatch, bit-exact with the reference's
    ``counting_scatter_expert_major_dispatch`` (DWDP/dispatcher/kernels/reference.py:163-257).
    With ``hidden`` it also gathers the packed bf16 activation rows."""
    _require_cuda(topk_indices, topk_weights, hidden)
    if topk_indices.shape != topk_weights.shape:
        raise ValueError("topk_indices and topk_weights must have identical shapes")
    if topk_indices.ndim < 1 or topk_indices.shape[-1] <= 0:
        raise ValueError("topk_indices must have a positive top-k dimension")
    if topk_indices.dtype.is_floating_point:
        raise ValueError("topk_indices must use an integer dtype")
    if not topk_weights.dtype.is_floating_point:
        raise ValueError("topk_weights must use a floating-point dtype")
    K = topk_indices.shape[-1]
    idx = topk_indices.reshape(-1).to(torch.int64).contiguous()
    wts = topk_weights.reshape(-1).contiguous()
    N = idx.numel()
    T = N // K
    dev = idx.device
    if out is None:
        out = DispatchResult(
            expert_counts=torch.empty(num_experts, dtype=torch.int64, device=dev),
            expert_offsets=torch.empty(num_experts + 1, dtype=torch.int64, device=dev),
            token_permutation=torch.empty(N, dtype=torch.int64, device=dev),
            inverse_permutation=torch.empty(N, dtype=torch.int64, device=dev),
            packed_expert_ids=torch.empty(N, dtype=torch.int64, device=dev),
            packed_token_indices=torch.empty(N, dtype=torch.int64, device=dev),
            packed_routing_weights=torch.empty(N, dtype=wts.dtype, device=dev),
            packed_hidden=None,
        )
    H = 0
    if hidden is not None:
        if hidden.dtype != torch.bfloat16:
            raise ValueError("packed activation gather expects bf16 hidden states")
        H = hidden.shape[-1]
        hidden = hidden.reshape(-1, H).contiguous()
        if out.packed_hidden is None:
            out.packed_hidden = torch.empty(N, H, dtype=torch.bfloat16, device=dev)
    if scratch is None:
        scratch = torch.empty(dispatch_scratch_bytes(T, K, num_experts), dtype=torch.uint8, device=dev)
    rc = _lib.load().dwdp_dispatch(
        idx.data_ptr(), wts.data_ptr(), dtype_code(wts.dtype), T, K, num_experts,
        _ptr(out.expert_counts), _ptr(out.expert_offsets), _ptr(out.token_permutation),
        _ptr(out.inverse_permutation), _ptr(out.packed_expert_ids), _ptr(out.packed_token_indices),
        _ptr(out.packed_routing_weights), _ptr(hidden), H,
        _ptr(out.packed_hidden) if hidden is not None else None, scratch.data_ptr(), _ptr(status),
        _stream(),
    )
    _lib.check(rc, "dispatch")
    return out


def gather_rows(hidden: torch.Tensor, token_index: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """packed[d] = hidden[token_index[d]] (bf16 rows)."""
    _require_cuda(hidden, token_index)
    if hidden.dtype != torch.bfloat16:
        raise ValueError("gather_rows expects bf16 hidden states")
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H).contiguous()
    idx = token_index.to(torch.int64).contiguous()
    if out is None:
        out = torch.empty(idx.numel(), H, dtype=torch.bfloat16, device=x.device)
    rc = _lib.load().dwdp_gather_rows(x.data_ptr(), idx.data_ptr(), idx.numel(), H, x.shape[0], out.data_ptr(),
                                      None, _stream())
    _lib.check(rc, "gather_rows")
    return out


def quantize_activations_blockwise(
    source: torch.Tensor, row_index: torch.Tensor | None = None, *, status: torch.Tensor | None = None,
    scale_layout: str = "rows",
) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's ``quantize_activations_blockwise`` (DWDP/executor/fp8.py:86-115) on
    the GPU: bf16 [M, K] -> (float8_e4m3fn [M, K], fp32 scales [M, K/128]), one scale per
    (row, 128 channels). ``row_index`` quantises source rows ``row_index[r]`` instead of
    row r; ``scale_layout="blocks"`` returns the scales transposed, [K/128, M]."""
    _require_cuda(source)
    if source.dtype != torch.bfloat16 or source.dim() != 2:
        raise ValueError("quantize_activations_blockwise expects a 2D bf16 [tokens, channels] tensor")
    if scale_layout not in ("rows", "blocks"):
        raise ValueError("scale_layout must be 'rows' or 'blocks'")
    x = source.contiguous()
    M0, K = x.shape
    idx = row_index.to(torch.int64).contiguous() if row_index is not None else None
    M = idx.numel() if idx is not None else M0
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    shape = (M, K // 128) if scale_layout == "rows" else (K // 128, M)
    sc = torch.empty(shape, dtype=torch.float32, device=x.device)
    rc = _lib.load().dwdp_quantize_activations_blockwise(
        x.data_ptr(), M0, _ptr(idx), M, K, q.data_ptr(), sc.data_ptr(), 0 if scale_layout == "rows" else 1,
        _ptr(status), _stream())
    _lib.check(rc, "quantize_activations_blockwise")
    return q, sc


def route_dispatch_small_fits(num_tokens: int, top_k: int, num_experts: int, hidden: torch.Tensor,
                              weight: torch.Tensor) -> bool:
    """Whether :func:`route_dispatch_small` covers this call (bf16, 0 < T*K <= 256, E <= 256)."""
    return (hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and 0 < num_tokens * top_k <= 256
            and num_experts <= 256 and top_k <= 16 and hidden.shape[-1] % 8 == 0)


# Token counts up to which the layers use route_dispatch_small: measured on the Qwen shape
# (K = 4, E = 60), layer time fused / unfused: T = 1 49.8 / 52.9 us, T = 4 64.9 / 65.4, T = 8
# 86.4 / 86.3, T = 64 180.8 / 130.0 (its last CTA's top-k and sort run serially).
FUSED_ROUTING_MAX_TOKENS = 4


def use_fused_routing(num_tokens: int, top_k: int, num_experts: int, hidden: torch.Tensor,
                      weight: torch.Tensor) -> bool:
    """The layers' choice: route_dispatch_small where it fits and T <= FUSED_ROUTING_MAX_TOKENS."""
    return num_tokens <= FUSED_ROUTING_MAX_TOKENS and route_dispatch_small_fits(num_tokens, top_k, num_experts,
                                                                                 hidden, weight)


def route_dispatch_small(hidden: torch.Tensor, weight: torch.Tensor, top_k: int, router: RouterResult,
                         disp: DispatchResult, ticket: torch.Tensor, gate_logit: torch.Tensor | None = None, *,
                         bias: torch.Tensor | None = None, shared_gate_weight: torch.Tensor | None = None,
                         score_scale: float = 1.0, renormalize: int | bool = True, eps: float = 1e-9,
                         status: torch.Tensor | None = None) -> None:
    """:func:`router_topk` then :func:`dispatch` (fp32 routing weights, no row gather) in ONE
    launch for decode-sized batches, into the given result holders. ``ticket`` is one int32 of
    device memory, zero before the first call (the kernel leaves it at zero)."""
    _require_cuda(hidden, weight, ticket, bias, shared_gate_weight)
    H = hidden.shape[-1]
    x = hidden.reshape(-1, H).contiguous()
    T = x.shape[0]
    E = weight.shape[0]
    if not route_dispatch_small_fits(T, top_k, E, x, weight):
        raise ValueError("route_dispatch_small needs bf16, 0 < T * K <= 256, E <= 256, K <= 16")
    if disp.packed_routing_weights.dtype != torch.float32:
        raise ValueError("route_dispatch_small writes fp32 packed routing weights")
    gw = shared_gate_weight.reshape(-1).to(weight.dtype).contiguous() if shared_gate_weight is not None else None
    if gw is not None and (gate_logit is None or router.shared_gate is None):
        raise ValueError("a shared gate weight needs gate_logit scratch and a shared_gate output")
    b = None if bias is None else bias.float().contiguous()
    rc = _lib.load().dwdp_route_dispatch_small(
        x.data_ptr(), weight.contiguous().data_ptr(), _ptr(b), _ptr(gw), T, H, E, top_k, float(score_scale),
        int(renormalize), float(eps), router.router_logits.data_ptr(), _ptr(gate_logit),
        _ptr(router.routing_probabilities), router.topk_indices.data_ptr(), router.topk_weights.data_ptr(),
        _ptr(router.shared_gate), disp.expert_counts.data_ptr(), disp.expert_offsets.data_ptr(),
        disp.token_permutation.data_ptr(), disp.inverse_permutation.data_ptr(), disp.packed_expert_ids.data_ptr(),
        disp.packed_token_indices.data_ptr(), disp.packed_routing_weights.data_ptr(), ticket.data_ptr(),
        _ptr(status), _stream())
    _lib.check(rc, "route_dispatch_small")


# --------------------------------------------------------------------------- schedule
@dataclass
class ScheduleResult:
    expert_queue: torch.Tensor
    expert_starts: torch.Tensor
    expert_ends: torch.Tensor
    expert_counts: torch.Tensor
    execution_priority: torch.Tensor
    stream_assignments: torch.Tensor
    num_active: torch.Tensor  # [1] int64 on device


def schedule(expert_counts: torch.Tensor, expert_offsets: torch.Tensor, stream_count: int = 1) -> ScheduleResult:
    """Ascending-expert round-robin schedule (DWDP/scheduler/ops/round_robin.py:8-80),
    padded to E rows with -1 so it needs no host synchronisation."""
    _require_cuda(expert_counts, expert_offsets)
    if stream_count <= 0:
        raise ValueError("stream_count must be > 0")
    E = expert_counts.numel()
    dev = expert_counts.device
    counts = expert_counts.to(torch.int64).contiguous()
    offsets = expert_offsets.to(torch.int64).contiguous()

    def mk() -> torch.Tensor:
        return torch.empty(E, dtype=torch.int64, device=dev)

    res = ScheduleResult(mk(), mk(), mk(), mk(), mk(), mk(), torch.empty(1, dtype=torch.int64, device=dev))
    rc = _lib.load().dwdp_schedule(
        counts.data_ptr(), offsets.data_ptr(), E, stream_count,
        res.expert_queue.data_ptr(), res.expert_starts.data_ptr(), res.expert_ends.data_ptr(),
        res.expert_counts.data_ptr(), res.execution_priority.data_ptr(),
        res.stream_assignments.data_ptr(), res.num_active.data_ptr(), _stream(),
    )
    _lib.check(rc, "schedule")
    return res


# --------------------------------------------------------------------------- weights
def packed_weight_bytes(rows: int, cols: int, num_mats: int, dtype: torch.dtype) -> int:
    return int(_lib.load().dwdp_packed_weight_bytes(rows, cols, num_mats, dtype_code(dtype)))


def packed_scale_floats(rows: int, cols: int, num_mats: int, scale_mode: int) -> int:
    return int(_lib.load().dwdp_packed_scale_floats(rows, cols, num_mats, scale_mode))


def pack_weights(
    mats: list[torch.Tensor], dst_dtype: torch.dtype, scale_mode: int
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Quantise (fp8) or convert (bf16) one or two [R, C] projections into the
    tiled store. Returns (tiles uint8, scales fp32 or None)."""
    _require_cuda(*mats)
    if not 1 <= len(mats) <= 2:
        raise ValueError("pack_weights takes one or two matrices")
    R, C = mats[0].shape
    for m in mats:
        if tuple(m.shape) != (R, C) or m.dtype != mats[0].dtype:
            raise ValueError("packed matrices must share shape and dtype")
    src = [m.contiguous() for m in mats]
    dev = src[0].device
    tiles = torch.empty(packed_weight_bytes(R, C, len(src), dst_dtype), dtype=torch.uint8, device=dev)
    nsc = packed_scale_floats(R, C, len(src), scale_mode) if dst_dtype == torch.float8_e4m3fn else 0
    scales = torch.empty(nsc, dtype=torch.float32, device=dev) if nsc else None
    ptrs = (ctypes.c_void_p * 2)(*([m.data_ptr() for m in src] + [0] * (2 - len(src))))
    rc = _lib.load().dwdp_pack_weights(
        ctypes.cast(ptrs, ctypes.c_void_p), dtype_code(src[0].dtype), R, C, len(src),
        dtype_code(dst_dtype), scale_mode, tiles.data_ptr(), _ptr(scales), _stream(),
    )
    _lib.check(rc, "pack_weights")
    return tiles, scales


def unpack_weights(
    tiles: torch.Tensor, scales: torch.Tensor | None, rows: int, cols: int, num_mats: int,
    dst_dtype: torch.dtype, scale_mode: int,
) -> torch.Tensor:
    """Dequantised fp32 view [num_mats, rows, cols] of a packed store (for checks)."""
    _require_cuda(tiles, scales)
    out = torch.empty(num_mats, rows, cols, dtype=torch.float32, device=tiles.device)
    rc = _lib.load().dwdp_unpack_weights(
        tiles.data_ptr(), _ptr(scales), rows, cols, num_mats, dtype_code(dst_dtype), scale_mode,
        out.data_ptr(), _stream(),
    )
    _lib.check(rc, "unpack_weights")
    return out


# --------------------------------------------------------------------------- experts + merge
def moe_shared_parts(num_tokens: int, shared_intermediate: int) -> int:
    """Partial [T, H] slabs the shared-expert output buffer must hold."""
    return int(_lib.load().dwdp_moe_shared_parts(num_tokens, shared_intermediate))


def moe_workspace_bytes(num_tokens: int, top_k: int, num_experts: int, intermediate: int,
                        shared_intermediate: int) -> int:
    return int(_lib.load().dwdp_moe_workspace_bytes(num_tokens, top_k, num_experts, intermediate,
                                                    shared_intermediate))


def moe_experts(
    routed: _lib.ExpertGroup,
    shared: _lib.ExpertGroup | None,
    packed_hidden: torch.Tensor | None,
    hidden: torch.Tensor,
    top_k: int,
    counts: torch.Tensor,
    offsets: torch.Tensor,
    packed_weights: torch.Tensor,
    shared_gate: torch.Tensor | None,
    weighted_out: torch.Tensor,
    shared_out: torch.Tensor | None,
    workspace: torch.Tensor,
    status: torch.Tensor | None = None,
    *,
    packed_token_indices: torch.Tensor | None = None,
) -> None:
    """Grouped tcgen05 expert GEMMs (gate/up + SwiGLU, down + routing weight).

    Routed rows come from ``packed_hidden`` or, when it is None, from
    ``hidden[packed_token_indices]`` read inside the kernels (no gathered copy)."""
    _require_cuda(packed_hidden, hidden, counts, offsets, packed_weights, weighted_out, workspace,
                  packed_token_indices)
    if packed_weights.dtype != torch.float32:
        raise ValueError("packed routing weights must be fp32 for the grouped GEMM")
    T = hidden.shape[0]
    lib = _lib.load()
    shared_ref = ctypes.byref(shared) if shared is not None else None
    tail = (T, top_k, counts.data_ptr(), offsets.data_ptr(), packed_weights.data_ptr(), _ptr(shared_gate),
            weighted_out.data_ptr(), _ptr(shared_out), workspace.data_ptr(), workspace.numel(), _ptr(status),
            _stream())
    if packed_hidden is not None:
        rc = lib.dwdp_moe_experts(ctypes.byref(routed), shared_ref, packed_hidden.data_ptr(), hidden.data_ptr(),
                                  *tail)
    else:
        if packed_token_indices is None or packed_token_indices.dtype != torch.int64:
            raise ValueError("moe_experts needs packed_hidden or int64 packed_token_indices")
        rc = lib.dwdp_moe_experts_indexed(ctypes.byref(routed), shared_ref, packed_token_indices.data_ptr(),
                                          hidden.data_ptr(), *tail)
    _lib.check(rc, "moe_experts")


def moe_shared_workspace_bytes(num_tokens: int, hidden_size: int, shared_intermediate_size: int) -> int:
    return int(_lib.load().dwdp_moe_shared_workspace_bytes(num_tokens, hidden_size, shared_intermediate_size))


def moe_shared_expert(shared: _lib.ExpertGroup, hidden: torch.Tensor, shared_out: torch.Tensor,
                      workspace: torch.Tensor, status: torch.Tensor | None = None, *,
                      shared_gate: torch.Tensor | None = None) -> None:
    """The shared expert alone: ``shared_out`` [parts, T, H] bf16 partials
    (``moe_shared_parts(T, Is)`` of them). Ungated by default (``merge(..., shared_gate=g)``
    applies the gate); with ``shared_gate`` [T] fp32 the down epilogue applies it, as
    :func:`moe_experts` does for its shared rows."""
    _require_cuda(hidden, shared_out, workspace, status, shared_gate)
    if shared_gate is not None and (shared_gate.dtype != torch.float32 or shared_gate.numel() < hidden.shape[0]):
        raise ValueError("shared_gate must be fp32 with one value per token")
    rc = _lib.load().dwdp_moe_shared_expert(
        ctypes.byref(shared), hidden.data_ptr(), hidden.shape[0], _ptr(shared_gate), shared_out.data_ptr(),
        workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(),
    )
    _lib.check(rc, "moe_shared_expert")


def merge(
    weighted: torch.Tensor,
    inverse_permutation: torch.Tensor,
    num_tokens: int,
    top_k: int,
    *,
    shared_out: torch.Tensor | None = None,
    shared_parts: int = 1,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    shared_gate: torch.Tensor | None = None,
) -> torch.Tensor:
    """Deterministic token-major merge (DWDP/merger/kernels/reference.py:6-27). With
    ``shared_gate`` the shared partials are ungated and scaled by it here."""
    _require_cuda(weighted, inverse_permutation, shared_out, shared_gate)
    if weighted.dtype != torch.bfloat16:
        raise ValueError("merge expects bf16 weighted rows")
    H = weighted.shape[-1]
    if out is None:
        out = torch.empty(num_tokens, H, dtype=out_dtype, device=weighted.device)
    lib = _lib.load()
    inv = inverse_permutation.contiguous()
    if shared_gate is not None:
        if shared_out is None or shared_gate.dtype != torch.float32:
            raise ValueError("a gated merge needs shared_out and an fp32 shared_gate")
        rc = lib.dwdp_merge_gated(
            weighted.data_ptr(), inv.data_ptr(), shared_out.data_ptr(), shared_parts, shared_gate.data_ptr(),
            num_tokens, top_k, H, out.data_ptr(), dtype_code(out.dtype), _stream(),
        )
    else:
        rc = lib.dwdp_merge(
            weighted.data_ptr(), inv.data_ptr(), _ptr(shared_out), shared_parts, num_tokens,
            top_k, H, out.data_ptr(), dtype_code(out.dtype), _stream(),
        )
    _lib.check(rc, "merge")
    return out


# --------------------------------------------------------------------------- decode-step attention pieces
def add_rmsnorm(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """residual += delta (in place, when delta is given); returns rmsnorm(residual) * weight
    (Qwen2MoeRMSNorm, fp32 arithmetic, bf16 rows)."""
    _require_cuda(residual, delta, weight)
    if residual.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("add_rmsnorm expects bf16 residual and weight")
    if not residual.is_contiguous() or (delta is not None and (not delta.is_contiguous()
                                                              or delta.shape != residual.shape)):
        raise ValueError("add_rmsnorm expects contiguous residual/delta of one shape")
    H = residual.shape[-1]
    if out is None:
        out = torch.empty_like(residual)
    rc = _lib.load().dwdp_add_rmsnorm(residual.data_ptr(), _ptr(delta), weight.data_ptr(), residual.numel() // H, H,
                                      float(eps), out.data_ptr(), _stream())
    _lib.check(rc, "add_rmsnorm")
    return out


def rope_append_kv(qkv: torch.Tensor, qkv_bias: torch.Tensor | None, positions: torch.Tensor,
                   block_table: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, rope_theta: float,
                   q_out: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """qkv [B, 3*NH*D] (+bias) -> rotated q [B, NH, D]; rotated k and v stored at
    positions[b] of the paged caches [num_blocks, block_size, NH, D]."""
    _require_cuda(qkv, qkv_bias, positions, block_table, k_cache, v_cache)
    if positions.dtype != torch.int32 or block_table.dtype != torch.int32:
        raise ValueError("positions and block_table must be int32")
    nb, bs, NH, D = k_cache.shape
    B = qkv.shape[0]
    if qkv.shape[-1] != 3 * NH * D or v_cache.shape != k_cache.shape:
        raise ValueError("qkv width must be 3 * num_heads * head_dim of the cache")
    if q_out is None:
        q_out = torch.empty(B, NH, D, dtype=torch.bfloat16, device=qkv.device)
    rc = _lib.load().dwdp_rope_append_kv(qkv.data_ptr(), _ptr(qkv_bias), positions.data_ptr(), block_table.data_ptr(),
                                         B, block_table.shape[-1], nb, NH, D, bs, float(rope_theta), q_out.data_ptr(),
                                         k_cache.data_ptr(), v_cache.data_ptr(), _ptr(status), _stream())
    _lib.check(rc, "rope_append_kv")
    return q_out


def paged_attention_splits(batch: int, num_heads: int, max_len: int, block_size: int = 16,
                           sm_count: int = 148) -> int:
    """Context chunks per sequence for ``paged_attention``. On the bulk-copy path (8, 16 or 32
    heads, block_size % 4 == 0) a CTA covers one chunk of one sequence for all heads and
    2 (16 heads), 4 (8) or 1 (32) CTAs fit on an SM: pick the split count, down to chunks of
    16 positions, whose CTA count fills whole waves best (the fewest splits within 2 % of the
    best; at B = 1 more splits measured faster than shorter combines). The
    fallback path (one CTA per (sequence, head, chunk)) asks for ~4 CTAs per SM."""
    if num_heads in (8, 16, 32) and block_size % 4 == 0:
        slots = sm_count * {8: 4, 16: 2, 32: 1}[num_heads]
        effs = []
        for s in range(1, max(1, max_len // 16) + 1):
            chunk = -(-(-(-max_len // s)) // 4) * 4
            ctas = batch * -(-max_len // chunk)
            effs.append((ctas / (-(-ctas // slots) * slots), s))
        top = max(e for e, _ in effs)
        return min(s for e, s in effs if e >= 0.98 * top)
    want = max(1, -(-4 * sm_count // max(1, batch * num_heads)))
    return max(1, min(want, -(-max_len // 64)))


def paged_attention_workspace(batch: int, num_heads: int, splits: int, device) -> torch.Tensor:
    n = _lib.load().dwdp_paged_attention_workspace_bytes(batch, num_heads, splits)
    return torch.empty(n, dtype=torch.uint8, device=device)


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                    seq_lens: torch.Tensor, max_len: int, *, splits: int | None = None, scale: float | None = None,
                    workspace: torch.Tensor | None = None, out: torch.Tensor | None = None,
                    status: torch.Tensor | None = None) -> torch.Tensor:
    """One-query paged attention: q [B, NH, D] over positions [0, seq_lens[b]) of each
    sequence's pages -> [B, NH, D] bf16. ``max_len`` bounds every seq_len (fixed per graph)."""
    _require_cuda(q, k_cache, v_cache, block_table, seq_lens)
    if seq_lens.dtype != torch.int32 or block_table.dtype != torch.int32:
        raise ValueError("seq_lens and block_table must be int32")
    B, NH, D = q.shape
    bs = k_cache.shape[1]
    if v_cache.shape != k_cache.shape:
        raise ValueError("k_cache and v_cache must have the same [num_blocks, block_size, NH, D] shape")
    splits = splits or paged_attention_splits(B, NH, max_len, bs)
    if workspace is None:
        workspace = paged_attention_workspace(B, NH, splits, q.device)
    if out is None:
        out = torch.empty(B, NH, D, dtype=torch.bfloat16, device=q.device)
    rc = _lib.load().dwdp_paged_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(),
                                          seq_lens.data_ptr(), B, block_table.shape[-1], k_cache.shape[0], NH, D, bs,
                                          int(max_len),
                                          splits, float(scale if scale is not None else D ** -0.5),
                                          workspace.data_ptr(), out.data_ptr(), _ptr(status), _stream())
    _lib.check(rc, "paged_attention")
    return out



# ----------------------------------------------------------------------------- TensorList
def tensor_list_build(plan_rows: tuple, plan_len: int, experts: _lib.ExpertGroup, bases: _lib.TensorListBases,
                      handle: _lib.TensorListHandle, meta: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """Fill ``handle.fields`` on the device from the plan rows (queue, starts, counts,
    priorities or None, streams or None); ``meta`` int64[2] receives (size, max_m)."""
    _require_cuda(meta, *[t for t in plan_rows if t is not None])
    for t in plan_rows:
        if t is not None and (t.dtype != torch.int64 or not t.is_contiguous()):
            raise ValueError("TensorList plan rows must be contiguous int64 tensors")
    lib = _lib.load()
    rc = lib.dwdp_tensor_list_build(*[_ptr(t) for t in plan_rows], plan_len, ctypes.byref(experts),
                                    ctypes.byref(bases), ctypes.byref(handle), meta.data_ptr(), _ptr(status),
                                    _stream())
    _lib.check(rc, "tensor_list_build")


def grouped_moe(handle: _lib.TensorListHandle, shared: _lib.ExpertGroup | None, packed_token_indices: torch.Tensor,
                hidden: torch.Tensor, top_k: int, packed_weights: torch.Tensor, shared_gate: torch.Tensor | None,
                weighted_out: torch.Tensor, shared_out: torch.Tensor | None, workspace: torch.Tensor,
                status: torch.Tensor | None = None) -> None:
    """Grouped expert GEMMs over the entries of a TensorList (``dwdp_grouped_moe``)."""
    _require_cuda(packed_token_indices, hidden, packed_weights, weighted_out, workspace)
    if packed_weights.dtype != torch.float32:
        raise ValueError("packed routing weights must be fp32 for the grouped GEMM")
    if packed_token_indices.dtype != torch.int64:
        raise ValueError("packed_token_indices must be int64")
    lib = _lib.load()
    rc = lib.dwdp_grouped_moe(ctypes.byref(handle), ctypes.byref(shared) if shared is not None else None,
                              packed_token_indices.data_ptr(), hidden.data_ptr(), hidden.shape[0], top_k,
                              packed_weights.data_ptr(), _ptr(shared_gate), weighted_out.data_ptr(), _ptr(shared_out),
                              workspace.data_ptr(), workspace.numel(), _ptr(status), _stream())
    _lib.check(rc, "grouped_moe")

"""``fused_moe`` with the reference's name and signature
(DWDP/executor/kernels/fused_moe.py:109-177) and correct semantics:

    out[t] = sum_k topk_weights[t, k] * down_e(silu(gate_e(x_t)) * up_e(x_t)),  e = topk_ids[t, k]

``w1`` holds gate and up stacked: ``[E, 2I, H]`` (gate rows then up rows, the
``FusedGateUpWeightView.materialize`` layout, DWDP/executor/weights.py:176-187)
or ``[E, H, 2I]`` (the reference kernel's indexing); ``w2`` is ``[E, H, I]`` or
``[E, I, H]``. When the shapes cannot tell the layouts apart (H == 2I for w1,
H == I for w2) pass ``layout="out_in"`` (nn.Linear ``[out, in]``) or
``layout="in_out"``. Unquantised (bf16/f16/f32) weights are converted once to
the packed bf16 store and cached by tensor identity and version; quantised
experts go through ExpertWeightStore. The routing is deterministic (a stable
counting sort instead of the reference's ``torch.sort``) and nothing reads
device values back to the host.
"""
from __future__ import annotations

import weakref

import torch

from . import ops
from .weights import ExpertWeightStore

# id(w1) -> (weak reference to w1, stamp, store); tensors cannot key a WeakKeyDictionary
# because their __eq__ is elementwise.
_CACHE: dict[int, tuple] = {}


def _split_w1(w1: torch.Tensor, H: int, layout: str | None) -> tuple[torch.Tensor, torch.Tensor]:
    _, a, b = w1.shape
    if layout is None:
        if a == b:
            raise ValueError("w1 is square ([E, H, 2I] with H == 2I is ambiguous); pass layout=")
        layout = "out_in" if b == H else "in_out"
    if layout == "out_in":  # [E, 2I, H]
        if b != H:
            raise ValueError(f"w1 [E, 2I, H] must have H={H} columns")
        I = a // 2
        return w1[:, :I], w1[:, I:]
    if layout == "in_out":  # [E, H, 2I]
        if a != H:
            raise ValueError(f"w1 [E, H, 2I] must have H={H} rows")
        I = b // 2
        return w1[:, :, :I].transpose(1, 2), w1[:, :, I:].transpose(1, 2)
    raise ValueError("layout must be 'out_in' or 'in_out'")


def _down(w2: torch.Tensor, H: int, I: int, layout: str | None) -> torch.Tensor:
    shape = tuple(w2.shape[1:])
    if layout == "out_in":
        if shape != (H, I):
            raise ValueError(f"w2 [E, H, I] must be [E, {H}, {I}]")
        return w2
    if layout == "in_out":
        if shape != (I, H):
            raise ValueError(f"w2 [E, I, H] must be [E, {I}, {H}]")
        return w2.transpose(1, 2)
    if layout is not None:
        raise ValueError("layout must be 'out_in' or 'in_out'")
    if H == I:
        raise ValueError("w2 is square ([E, H, I] with H == I is ambiguous); pass layout=")
    if shape == (H, I):
        return w2
    if shape == (I, H):
        return w2.transpose(1, 2)
    raise ValueError(f"w2 must be [E, {H}, {I}] or [E, {I}, {H}]")


def _store_for(w1: torch.Tensor, w2: torch.Tensor, H: int, layout: str | None) -> ExpertWeightStore:
    hit = _CACHE.get(id(w1))
    stamp = (w1._version, w2._version, w2.data_ptr(), layout)
    if hit is not None and hit[0]() is w1 and hit[1] == stamp:
        return hit[2]
    if w1.dtype == torch.float8_e4m3fn or w2.dtype == torch.float8_e4m3fn:
        raise ValueError("fused_moe takes unquantised weights; quantised experts go through ExpertWeightStore")
    gate, up = _split_w1(w1, H, layout)
    I = gate.shape[1]
    down = _down(w2, H, I, layout)
    E = w1.shape[0]
    store = ExpertWeightStore(E, H, I, weight_dtype=torch.bfloat16, device=w1.device)
    for e in range(E):
        store.load_expert(e, gate[e].contiguous(), up[e].contiguous(), down[e].contiguous())
    key = id(w1)
    _CACHE[key] = (weakref.ref(w1, lambda _r, k=key: _CACHE.pop(k, None)), stamp, store)
    return store


def fused_moe(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, topk_ids: torch.Tensor,
              topk_weights: torch.Tensor, *, layout: str | None = None) -> torch.Tensor:
    """[T, H] hidden, stacked expert weights, [T, K] routing -> [T, H] (hidden dtype)."""
    if hidden_states.ndim != 2:
        raise ValueError("hidden_states must be [num_tokens, hidden_dim]")
    if topk_ids.shape != topk_weights.shape or topk_ids.ndim != 2 or topk_ids.shape[0] != hidden_states.shape[0]:
        raise ValueError("topk_ids and topk_weights must both be [num_tokens, top_k]")
    T, H = hidden_states.shape
    K = topk_ids.shape[1]
    out_dtype = hidden_states.dtype
    if T == 0:
        return torch.zeros_like(hidden_states)
    store = _store_for(w1, w2, H, layout)
    x = hidden_states.to(torch.bfloat16).contiguous()
    disp = ops.dispatch(topk_ids, topk_weights.float(), store.num_experts, hidden=x)
    ws = torch.empty(ops.moe_workspace_bytes(T, K, store.num_experts, store.intermediate_size, 0),
                     dtype=torch.uint8, device=x.device)
    weighted = torch.empty(T * K, H, dtype=torch.bfloat16, device=x.device)
    ops.moe_experts(store.group(), None, disp.packed_hidden, x, K, disp.expert_counts, disp.expert_offsets,
                    disp.packed_routing_weights, None, weighted, None, ws)
    out = ops.merge(weighted, disp.inverse_permutation, T, K,
                    out_dtype=torch.float32 if out_dtype == torch.float32 else torch.bfloat16)
    return out if out.dtype == out_dtype else out.to(out_dtype)

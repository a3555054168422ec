"""TensorList: the non-owning structure-of-arrays descriptor of the active experts
(DWDP/executor/tensor_list.py:29-228), with the reference's fields in its order.

Every field is a contiguous int64 device row of ``capacity`` entries inside one
buffer owned by a :class:`TensorListWorkspace` (the reference's
``ExecutorWorkspace`` role, executor/workspace.py:9-64). Pointer fields hold raw
device addresses and keep nothing alive; a descriptor is valid for the forward
call whose tensors it describes.

Where the reference fills the fields on the host (one pass over the plan, a
pinned H2D copy, a stream sync and ``.item()`` for ``max_m``,
tensor_list.py:69-198), ``from_plans`` fills them with ONE kernel launch
(``dwdp_tensor_list_build``) that compacts the plan's active rows on the device.
``size`` and ``launch_dimensions`` are host ints as in the reference, read back
with one 16-byte copy; ``sync=False`` skips that read (``size`` then reports the
capacity: entries past the active count are empty, count 0, and every consumer
skips them), so the fill can be captured in a CUDA graph.

B200-specific meaning of a few fields:
* ``gate_weight_ptrs`` and ``up_weight_ptrs`` both name the expert's packed
  gate/up slab (the row block's gate tiles, then its up tiles);
* ``quantization_ptrs`` is the gate/up scale address (the reference leaves it 0,
  tensor_list.py:160) and the extra row ``down_quantization_ptrs`` the down
  scales; both 0 for bf16 weights;
* ``gate_ld``/``up_ld``/``down_ld`` are the nn.Linear row strides (H, H, I) of
  the unpacked weights the packed tiles were made from.

``grouped_moe`` runs the grouped tcgen05 GEMMs straight from the descriptor's
rows (``dwdp_grouped_moe``): entry i plays the role of expert i.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, ops

FIELD_NAMES = (
    "input_ptrs", "token_index_ptrs", "routing_weight_ptrs", "gate_weight_ptrs", "up_weight_ptrs",
    "down_weight_ptrs", "intermediate_ptrs", "output_ptrs", "weighted_output_ptrs", "quantization_ptrs",
    "expert_ids", "token_offsets", "token_counts", "m", "n", "k", "intermediate_n", "input_ld", "gate_ld",
    "up_ld", "down_ld", "output_ld", "dtype_codes", "workspace_indices", "execution_priorities", "stream_ids",
)
EXTRA_FIELD_NAMES = ("down_quantization_ptrs",)
MAX_CAPACITY = 1024


class TensorListWorkspace:
    """Owns the reusable field buffer ([27, capacity] int64), the (size, max_m) pair
    and a device status word. Capacity grows on demand and never shrinks, like the
    reference's ``ensure_tensorlist_capacity`` (executor/workspace.py)."""

    def __init__(self, device: torch.device | str = "cuda", capacity: int = 0) -> None:
        self.device = torch.device(device)
        self.capacity = 0
        self.fields: torch.Tensor | None = None
        self.meta = torch.zeros(2, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        if capacity:
            self.ensure_capacity(capacity)

    def ensure_capacity(self, n: int) -> int:
        if n > MAX_CAPACITY:
            raise ValueError(f"TensorList capacity {n} exceeds {MAX_CAPACITY} entries")
        if n > self.capacity:
            self.capacity = max(n, 1)
            self.fields = torch.zeros(_lib.TL_ROWS, self.capacity, dtype=torch.int64, device=self.device)
        return self.capacity


@dataclass(slots=True)
class TensorList:
    size: int
    capacity: int
    input_ptrs: torch.Tensor
    token_index_ptrs: torch.Tensor
    routing_weight_ptrs: torch.Tensor
    gate_weight_ptrs: torch.Tensor
    up_weight_ptrs: torch.Tensor
    down_weight_ptrs: torch.Tensor
    intermediate_ptrs: torch.Tensor
    output_ptrs: torch.Tensor
    weighted_output_ptrs: torch.Tensor
    quantization_ptrs: torch.Tensor
    expert_ids: torch.Tensor
    token_offsets: torch.Tensor
    token_counts: torch.Tensor
    m: torch.Tensor
    n: torch.Tensor
    k: torch.Tensor
    intermediate_n: torch.Tensor
    input_ld: torch.Tensor
    gate_ld: torch.Tensor
    up_ld: torch.Tensor
    down_ld: torch.Tensor
    output_ld: torch.Tensor
    dtype_codes: torch.Tensor
    workspace_indices: torch.Tensor
    execution_priorities: torch.Tensor
    stream_ids: torch.Tensor
    launch_dimensions: tuple[int, int, int]
    down_quantization_ptrs: torch.Tensor | None = None
    handle: _lib.TensorListHandle | None = None  # what dwdp_grouped_moe takes

    @classmethod
    def from_plans(cls, hidden_states: torch.Tensor, dispatch_plan, execution_plan, workspace: TensorListWorkspace,
                   provider, packed_outputs: torch.Tensor | None, weighted_outputs: torch.Tensor | None,
                   intermediate: torch.Tensor | None, *, sync: bool = True) -> "TensorList":
        """Build the descriptor from the finished plans (tensor_list.py:69-198). ``provider``
        is an ``ExpertWeightStore`` (any object with ``group()``, ``hidden_size`` and
        ``intermediate_size``). Raises ``ValueError`` on the reference's contract violations."""
        dev = hidden_states.device
        H = provider.hidden_size
        if hidden_states.dim() != 2 or hidden_states.shape[1] != H:
            raise ValueError("provider hidden size does not match activations")
        if packed_outputs is not None and weighted_outputs is not None and packed_outputs.shape != weighted_outputs.shape:
            raise ValueError("packed and weighted output buffers must have the same shape")
        asg = dispatch_plan.assignments
        ep = execution_plan
        for name, t in (("packed token indices", asg.packed_token_indices),
                        ("routing weights", asg.packed_routing_weights), ("expert queue", ep.expert_queue),
                        ("expert starts", ep.expert_starts), ("expert counts", ep.expert_counts)):
            if t.device != dev:
                raise ValueError(f"TensorList {name} must share the activation device")
        plan_len = int(ep.expert_queue.numel())
        cap = workspace.ensure_capacity(max(plan_len, 1))
        group = provider.group()
        out_like = weighted_outputs if weighted_outputs is not None else packed_outputs

        def row_bytes(t):
            return 0 if t is None else t.stride(0) * t.element_size()

        b = _lib.TensorListBases()
        b.input, b.token_index = hidden_states.data_ptr(), asg.packed_token_indices.data_ptr()
        b.routing_weights = asg.packed_routing_weights.data_ptr()
        b.intermediate = ops._ptr(intermediate)
        b.output, b.weighted_output = ops._ptr(packed_outputs), ops._ptr(weighted_outputs)
        b.intermediate_row_bytes, b.output_row_bytes = row_bytes(intermediate), row_bytes(packed_outputs)
        b.weighted_row_bytes = row_bytes(weighted_outputs)
        b.n = out_like.shape[1] if out_like is not None else H
        b.k = H
        b.intermediate_n = intermediate.shape[1] if intermediate is not None else provider.intermediate_size
        b.input_ld = hidden_states.stride(0)
        b.gate_ld = b.up_ld = H
        b.down_ld = provider.intermediate_size
        b.output_ld = out_like.stride(0) if out_like is not None else H
        b.dtype_code = ops.dtype_code(hidden_states.dtype)
        h = _lib.TensorListHandle()
        h.capacity, h.fields = cap, workspace.fields.data_ptr()
        h.hidden_size, h.intermediate_size = H, provider.intermediate_size
        h.weight_dtype, h.scale_mode, h.act_quant = group.weight_dtype, group.scale_mode, group.act_quant
        rows = tuple(t.contiguous() if t is not None else None for t in (
            ep.expert_queue, ep.expert_starts, ep.expert_counts, ep.execution_priority, ep.stream_assignments))
        workspace.status.zero_()
        ops.tensor_list_build(rows, plan_len, group, b, h, workspace.meta, workspace.status)
        if sync:
            size, max_m = (int(v) for v in workspace.meta.tolist())
            st = workspace.status.tolist()
            if st[0] != 0:
                raise RuntimeError(f"TensorList build: device status {st}")
        else:
            size, max_m = cap, 0
        f = workspace.fields
        views = {name: f[i, :size] for i, name in enumerate(FIELD_NAMES)}
        return cls(size=size, capacity=cap, launch_dimensions=(max_m, int(b.n), int(b.intermediate_n)),
                   down_quantization_ptrs=f[len(FIELD_NAMES), :size], handle=h, **views)


def grouped_moe(tl: TensorList, hidden: torch.Tensor, dispatch_plan, weighted_out: torch.Tensor,
                moe_workspace: torch.Tensor, *, top_k: int | None = None, shared=None,
                shared_gate: torch.Tensor | None = None, shared_out: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> torch.Tensor:
    """Run the grouped expert GEMMs the TensorList describes (``dwdp_grouped_moe``):
    ``weighted_out[r] = w[r] * down(silu(gate(x)) * up(x))`` for every packed row r of
    every entry, x = ``hidden[packed_token_indices[r]]``. ``moe_workspace`` must hold
    ``ops.moe_workspace_bytes(T, K, tl.capacity, I, Is)`` bytes."""
    if tl.handle is None:
        raise ValueError("TensorList was not built by TensorList.from_plans")
    asg = dispatch_plan.assignments
    K = top_k if top_k is not None else dispatch_plan.metadata.top_k
    w = asg.packed_routing_weights
    if w.dtype != torch.float32:
        w = w.float()
    ops.grouped_moe(tl.handle, shared, asg.packed_token_indices, hidden, K, w, shared_gate, weighted_out,
                    shared_out, moe_workspace, status)
    return weighted_out


__all__ = ["TensorList", "TensorListWorkspace", "grouped_moe", "FIELD_NAMES"]

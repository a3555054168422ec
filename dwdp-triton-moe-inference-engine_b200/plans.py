"""The reference's stage-output dataclasses, restated with the same field names
and meaning (the drop-in contract between stages):

* ``RouterOutput``, ``RoutingMetadata``   — DWDP/router/types.py:10-18, router/metadata.py:12-26
* ``ExpertAssignments``, ``DispatchMetadata``, ``DispatchPlan``
                                           — DWDP/dispatcher/assignments.py, metadata.py, plan.py:9-14
* ``ExecutionPlan``                        — DWDP/scheduler/execution.py:22-38 (tensor fields; the
  per-expert rows are padded to E with -1 and ``num_active`` is a device scalar,
  so building the plan needs no host synchronisation)
* ``CommunicationPlan``                    — DWDP/comms_planner/metadata.py:107-125 (the two
  expert-id tensors and the policy name the executor reads)
* ``ExecutorOutput``, ``MergerOutput``     — DWDP/executor/outputs.py:62-82, merger/outputs.py:10-20

All integer tensors are int64, as the reference requires (dispatcher/config.py:23-26).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(slots=True)
class RoutingMetadata:
    num_tokens: int
    num_experts: int
    top_k: int
    tokens_per_expert: torch.Tensor | None = None
    expert_offsets: torch.Tensor | None = None
    flattened_token_indices: torch.Tensor | None = None
    flattened_expert_indices: torch.Tensor | None = None
    flattened_weights: torch.Tensor | None = None


@dataclass(slots=True)
class RouterOutput:
    router_logits: torch.Tensor
    routing_probabilities: torch.Tensor
    topk_indices: torch.Tensor
    topk_weights: torch.Tensor
    metadata: RoutingMetadata | None = None
    shared_gate: torch.Tensor | None = None  # sigmoid shared-expert gate when requested


@dataclass(slots=True)
class ExpertAssignments:
    expert_ids: torch.Tensor
    packed_token_indices: torch.Tensor
    packed_routing_weights: torch.Tensor


@dataclass(slots=True)
class DispatchMetadata:
    num_tokens: int
    num_assignments: int
    num_experts: int
    top_k: int
    token_shape: tuple[int, ...]
    expert_counts: torch.Tensor
    expert_offsets: torch.Tensor
    token_permutation: torch.Tensor
    inverse_permutation: torch.Tensor
    destination_positions: torch.Tensor
    stable_order: bool
    algorithm: str


@dataclass(slots=True)
class DispatchPlan:
    assignments: ExpertAssignments
    metadata: DispatchMetadata
    packed_hidden: torch.Tensor | None = None  # bf16 [T*K, H] rows in expert-major order, when gathered


@dataclass(slots=True)
class ExecutionPlan:
    execution_order: torch.Tensor
    expert_queue: torch.Tensor
    expert_starts: torch.Tensor
    expert_ends: torch.Tensor
    expert_counts: torch.Tensor
    execution_priority: torch.Tensor
    stream_assignments: torch.Tensor
    num_active: torch.Tensor
    scheduling_policy: str = "round_robin"
    deterministic: bool = True
    batches: tuple = ()

    def materialize(self) -> "ExecutionPlan":
        """The reference's variable-length form (drops the -1 padding; syncs the host)."""
        n = int(self.num_active.item())
        cut = lambda t: t[:n]  # noqa: E731
        return ExecutionPlan(cut(self.execution_order), cut(self.expert_queue), cut(self.expert_starts),
                             cut(self.expert_ends), cut(self.expert_counts), cut(self.execution_priority),
                             cut(self.stream_assignments), self.num_active, self.scheduling_policy,
                             self.deterministic, self.batches)


@dataclass(slots=True)
class CommunicationPlan:
    local_expert_ids: torch.Tensor
    remote_expert_ids: torch.Tensor
    planner_policy: str = "static"
    prefetch_buffer: int = 0
    cost_model: object | None = None  # cost_model.CommunicationCostModel for remote transfers


@dataclass(slots=True)
class ExecutorOutput:
    packed_expert_outputs: torch.Tensor | None
    weighted_expert_outputs: torch.Tensor | None
    backend: str
    deterministic: bool
    inverse_permutation: torch.Tensor | None = None
    token_shape: tuple[int, ...] = ()
    top_k: int = 1
    merged_expert_outputs: torch.Tensor | None = None
    expert_outputs: tuple = field(default_factory=tuple)


@dataclass(slots=True)
class MergerOutput:
    hidden_states: torch.Tensor
    backend: str
    deterministic: bool

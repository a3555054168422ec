"""The reference's stage-output dataclasses, restated with the same field names
and meaning (the drop-in contract between stages):

* ``RouterOutput``, ``RoutingMetadata``   — DWDP/router/types.py:10-18, router/metadata.py:12-26
* ``ExpertAssignments``, ``DispatchMetadata``, ``DispatchPlan``
                                           — DWDP/dispatcher/assignments.py, metadata.py, plan.py:9-14
* ``ExecutionPlan`` (+ batch, synchronisation, dependency metadata)
                                           — DWDP/scheduler/execution.py:10-38, metadata.py:8-38 (the
  per-expert rows are padded to E with -1 and ``num_active`` is a device scalar,
  so building the plan needs no host synchronisation; statistics are read lazily)
* ``CommunicationPlan``                    — DWDP/comms_planner/metadata.py:107-125, every field
  (its parts in :mod:`comms_metadata`)
* ``ExecutorOutput`` (+ ExpertOutput, OutputMetadata, ExecutionMetadata, timing and
  workspace metadata), ``MergerOutput`` (+ merge metadata and statistics)
                                           — DWDP/executor/outputs.py:10-82, executor/metadata.py,
                                             merger/outputs.py:10-20, merger/metadata.py

All integer tensors are int64, as the reference requires (dispatcher/config.py:23-26).
"""
from __future__ import annotations

from dataclasses import dataclass

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


# ----------------------------------------------------------------------------- scheduler
@dataclass(slots=True)
class ExecutionBatch:
    """DWDP/scheduler/execution.py:10-19."""

    expert_id: int
    start: int
    end: int
    count: int
    priority: int
    stream_id: int


@dataclass(slots=True)
class SynchronizationMetadata:
    """DWDP/scheduler/metadata.py:8-15."""

    barrier_after_batch: torch.Tensor
    cuda_event_ids: torch.Tensor | None = None
    stream_waits: torch.Tensor | None = None


@dataclass(slots=True)
class DependencyMetadata:
    """DWDP/scheduler/metadata.py:18-26."""

    dependency_src: torch.Tensor
    dependency_dst: torch.Tensor
    prefetch_expert_ids: torch.Tensor | None = None
    communication_groups: torch.Tensor | None = None


class LazyStatistics:
    """Statistics whose values live on the device: read an attribute and the values are
    copied to the host once (a synchronisation). Building the plan never synchronises, so a
    plan whose statistics nobody reads stays graph-capturable."""

    def __init__(self, compute, fields: tuple[str, ...]) -> None:
        self._compute = compute
        self._fields = fields
        self._values: dict | None = None

    def __getattr__(self, name: str):
        if name.startswith("_"):
            raise AttributeError(name)
        if self._values is None:
            self._values = self._compute()
        try:
            return self._values[name]
        except KeyError as exc:
            raise AttributeError(name) from exc

    def __repr__(self) -> str:
        return f"LazyStatistics({', '.join(self._fields)})"


SCHEDULER_STATISTICS_FIELDS = ("num_experts", "num_active_experts", "num_empty_experts", "num_execution_batches",
                               "num_assignments", "max_tokens_per_expert", "min_tokens_per_active_expert",
                               "scheduling_policy")


@dataclass(slots=True)
class ExecutionPlan:
    """DWDP/scheduler/execution.py:22-38, every field, plus ``num_active`` (a device scalar).
    The per-expert rows are padded to E with -1 (count -1 < 1, which the reference's executors
    skip), so the plan is built without reading the number of active experts back."""

    execution_order: torch.Tensor
    expert_queue: torch.Tensor
    expert_starts: torch.Tensor
    expert_ends: torch.Tensor
    expert_counts: torch.Tensor
    execution_priority: torch.Tensor
    stream_assignments: torch.Tensor
    batches: tuple = ()
    synchronization: SynchronizationMetadata | None = None
    dependencies: DependencyMetadata | None = None
    statistics: object | None = None
    scheduling_policy: str = "round_robin"
    deterministic: bool = True
    num_active: torch.Tensor | None = None

    def materialize(self) -> "ExecutionPlan":
        """The reference's variable-length form (drops the -1 padding; syncs the host)."""
        n = int(self.num_active.item()) if self.num_active is not None else int((self.expert_counts > 0).sum())
        cut = lambda t: t[:n]  # noqa: E731
        return ExecutionPlan(cut(self.execution_order), cut(self.expert_queue), cut(self.expert_starts),
                             cut(self.expert_ends), cut(self.expert_counts), cut(self.execution_priority),
                             cut(self.stream_assignments), self.batches, self.synchronization, self.dependencies,
                             self.statistics, self.scheduling_policy, self.deterministic, self.num_active)


from .comms_metadata import CommunicationPlan  # noqa: E402  (DWDP/comms_planner/metadata.py:107-125)


# ----------------------------------------------------------------------------- executor
@dataclass(slots=True)
class ExpertOutput:
    """DWDP/executor/outputs.py:10-19."""

    expert_id: int
    start: int
    end: int
    count: int
    priority: int
    stream_id: int


@dataclass(slots=True)
class OutputMetadata:
    """DWDP/executor/outputs.py:35-45: what the merger reads."""

    packed_token_indices: torch.Tensor
    packed_expert_ids: torch.Tensor
    packed_routing_weights: torch.Tensor
    token_permutation: torch.Tensor
    inverse_permutation: torch.Tensor
    token_shape: tuple[int, ...]
    top_k: int


@dataclass(slots=True)
class ExecutionMetadata:
    """DWDP/executor/outputs.py:48-59."""

    execution_order: torch.Tensor
    expert_queue: torch.Tensor
    expert_starts: torch.Tensor
    expert_ends: torch.Tensor
    stream_assignments: torch.Tensor
    communication_remote_expert_ids: torch.Tensor
    communication_policy: str
    scheduling_policy: str


EXECUTION_STATISTICS_FIELDS = ("num_executed_experts", "num_skipped_experts", "num_input_tokens", "num_assignments",
                               "hidden_size", "output_size", "backend")


@dataclass(slots=True)
class TimingMetadata:
    """DWDP/executor/metadata.py:8-13 (the merger's variant adds reduction_duration_us)."""

    expert_durations_us: torch.Tensor | None = None
    total_duration_us: float | None = None
    reduction_duration_us: float | None = None


@dataclass(slots=True)
class WorkspaceMetadata:
    """DWDP/executor/metadata.py:16-21, merger/metadata.py:40-45."""

    used_workspace: bool
    workspace_bytes: int


@dataclass(slots=True)
class ExecutorOutput:
    """DWDP/executor/outputs.py:62-82, every field in the reference's order. The merge inputs
    (inverse permutation, token shape, top-k) are read from ``output_metadata``."""

    packed_expert_outputs: torch.Tensor | None
    weighted_expert_outputs: torch.Tensor | None
    expert_outputs: tuple
    output_metadata: OutputMetadata
    execution_metadata: ExecutionMetadata | None
    statistics: object | None
    timing: TimingMetadata
    workspace: WorkspaceMetadata
    backend: str
    deterministic: bool
    merged_expert_outputs: torch.Tensor | None = None

    @property
    def inverse_permutation(self) -> torch.Tensor:
        return self.output_metadata.inverse_permutation

    @property
    def token_shape(self) -> tuple[int, ...]:
        return self.output_metadata.token_shape

    @property
    def top_k(self) -> int:
        return self.output_metadata.top_k


# ----------------------------------------------------------------------------- merger
@dataclass(slots=True)
class MergeMetadata:
    """DWDP/merger/metadata.py:20-28."""

    token_shape: tuple[int, ...]
    assignment_shape: tuple[int, int]
    inverse_permutation: torch.Tensor
    top_k: int
    deterministic: bool


@dataclass(slots=True)
class MergeStatistics:
    """DWDP/merger/metadata.py:8-17."""

    num_tokens: int
    num_assignments: int
    top_k: int
    output_size: int
    used_weighted_executor_outputs: bool
    backend: str


@dataclass(slots=True)
class MergerOutput:
    """DWDP/merger/outputs.py:10-20."""

    hidden_states: torch.Tensor
    metadata: MergeMetadata | None
    statistics: MergeStatistics | None
    timing: TimingMetadata
    workspace: WorkspaceMetadata
    backend: str
    deterministic: bool

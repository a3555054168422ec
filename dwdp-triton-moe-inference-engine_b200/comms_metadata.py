"""The communication plan's dataclasses, with the reference's names, fields and field
order (DWDP/comms_planner/metadata.py:12-125, graph.py, topology.py): the contract
between the communication planner, the engine that executes the plan and the executor
that reads ``local_expert_ids`` / ``remote_expert_ids``.

Only ``CommunicationPlan`` gains a field of its own after the reference's ones
(``prefetch_buffer``: the staging buffer the plan's copies land in).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(slots=True)
class CommunicationDescriptor:
    """One planned copy: bytes [start, end) of expert ``source_expert_id``'s slab on
    ``source_gpu`` into the same offsets of its staging slot on ``destination_gpu``."""

    descriptor_id: int
    op_type: str
    source_gpu: int
    destination_gpu: int
    source_expert_id: int
    destination_expert_id: int
    start: int
    end: int
    count: int
    priority: int
    stream_id: int


@dataclass(slots=True)
class TransferDescriptor:
    transfer_id: int
    descriptor_id: int
    source_gpu: int
    destination_gpu: int
    source_expert_id: int
    destination_expert_id: int
    estimated_bytes: int
    priority: int


@dataclass(slots=True)
class CommunicationGroup:
    group_id: int
    descriptor_ids: torch.Tensor
    source_gpu: int
    destination_gpu: int
    domain_id: int
    priority: int


@dataclass(slots=True)
class SynchronizationMetadata:
    barrier_node_ids: torch.Tensor
    cuda_event_ids: torch.Tensor
    stream_wait_edges: torch.Tensor
    synchronization_points: torch.Tensor


@dataclass(slots=True)
class DependencyMetadata:
    dependency_src: torch.Tensor
    dependency_dst: torch.Tensor
    dependency_type: torch.Tensor


@dataclass(slots=True)
class PrefetchPlan:
    prefetch_expert_ids: torch.Tensor
    prefetch_priorities: torch.Tensor
    prefetch_windows_us: torch.Tensor


@dataclass(slots=True)
class OverlapPlan:
    communication_node_ids: torch.Tensor
    compute_batch_ids: torch.Tensor
    overlap_windows_us: torch.Tensor


@dataclass(slots=True)
class CommunicationStatistics:
    num_local_experts: int
    num_remote_experts: int
    num_communication_nodes: int
    num_communication_edges: int
    num_transfer_descriptors: int
    num_communication_groups: int
    total_estimated_bytes: int
    total_estimated_latency_us: float
    planner_policy: str


@dataclass(slots=True)
class CommunicationNode:
    node_id: int
    descriptor_id: int
    op_type: str
    source_gpu: int
    destination_gpu: int
    expert_id: int
    priority: int
    stream_id: int


@dataclass(slots=True)
class CommunicationEdge:
    source_node_id: int
    destination_node_id: int
    dependency_type: str


@dataclass(slots=True)
class CommunicationGraph:
    nodes: tuple
    edges: tuple
    node_ids: torch.Tensor
    edge_src: torch.Tensor
    edge_dst: torch.Tensor

    @property
    def is_empty(self) -> bool:
        return len(self.nodes) == 0 and len(self.edges) == 0


@dataclass(slots=True)
class CommunicationDomain:
    domain_id: int
    domain_type: str
    gpu_ids: tuple
    bandwidth_gbps: float
    latency_us: float


@dataclass(slots=True)
class TopologyMetadata:
    local_gpu_id: int
    world_size: int
    local_rank: int
    gpu_ids: torch.Tensor
    numa_domains: torch.Tensor
    nvlink_connectivity: torch.Tensor | None
    nvswitch_domains: torch.Tensor | None
    pcie_hierarchy: torch.Tensor | None
    communication_domains: tuple
    locality_groups: tuple
    fabric: str
    default_link_bandwidth_gbps: float
    default_link_latency_us: float


@dataclass(slots=True)
class CommunicationPlan:
    local_expert_ids: torch.Tensor
    remote_expert_ids: torch.Tensor
    graph: CommunicationGraph | None = None
    communication_descriptors: tuple = ()
    transfer_descriptors: tuple = ()
    communication_groups: tuple = ()
    topology: TopologyMetadata | None = None
    synchronization: SynchronizationMetadata | None = None
    dependencies: DependencyMetadata | None = None
    prefetch: PrefetchPlan | None = None
    overlap: OverlapPlan | None = None
    cost_model: object | None = None  # cost_model.CommunicationCostModel
    statistics: CommunicationStatistics | None = None
    planner_policy: str = "static"
    deterministic: bool = True
    prefetch_buffer: int = 0

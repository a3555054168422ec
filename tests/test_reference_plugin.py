"""The drop-in boundary against the reference's own types and registries (CPU): every
field of the reference's stage-output dataclasses exists on this package's, and the B200
stages register into the reference's registries and are built by its builders."""
from __future__ import annotations

import dataclasses

import pytest
import torch

from tests.reference_import import import_reference

DWDP = import_reference()
pytestmark = pytest.mark.skipif(DWDP is None, reason="the reference package is not present")

PAIRS = [
    ("DWDP.router.types", "RouterOutput"),
    ("DWDP.router.metadata", "RoutingMetadata"),
    ("DWDP.dispatcher.plan", "DispatchPlan"),
    ("DWDP.dispatcher.assignments", "ExpertAssignments"),
    ("DWDP.dispatcher.metadata", "DispatchMetadata"),
    ("DWDP.scheduler.execution", "ExecutionPlan"),
    ("DWDP.scheduler.execution", "ExecutionBatch"),
    ("DWDP.scheduler.metadata", "SynchronizationMetadata"),
    ("DWDP.scheduler.metadata", "DependencyMetadata"),
    ("DWDP.executor.outputs", "ExecutorOutput"),
    ("DWDP.executor.outputs", "ExpertOutput"),
    ("DWDP.executor.outputs", "OutputMetadata"),
    ("DWDP.executor.outputs", "ExecutionMetadata"),
    ("DWDP.executor.metadata", "WorkspaceMetadata"),
    ("DWDP.merger.outputs", "MergerOutput"),
    ("DWDP.merger.metadata", "MergeMetadata"),
    ("DWDP.merger.metadata", "MergeStatistics"),
]


@pytest.mark.parametrize("module,name", PAIRS)
def test_dataclass_fields_cover_the_reference(pkg, module, name):
    import importlib

    ref = getattr(importlib.import_module(module), name)
    ours = getattr(pkg.plans, name)
    ref_fields = [f.name for f in dataclasses.fields(ref)]
    our_fields = [f.name for f in dataclasses.fields(ours)]
    missing = [f for f in ref_fields if f not in our_fields]
    assert not missing, f"{name}: fields of the reference missing here: {missing}"
    # the reference's fields keep their order (positional construction stays valid)
    assert [f for f in our_fields if f in ref_fields] == ref_fields


def test_statistics_fields_cover_the_reference(pkg):
    from DWDP.executor.outputs import ExecutionStatistics
    from DWDP.scheduler.metadata import SchedulerStatistics

    assert [f.name for f in dataclasses.fields(SchedulerStatistics)] == list(pkg.plans.SCHEDULER_STATISTICS_FIELDS)
    assert [f.name for f in dataclasses.fields(ExecutionStatistics)] == list(pkg.plans.EXECUTION_STATISTICS_FIELDS)


def test_register_with_reference_and_build(pkg):
    from DWDP.dispatcher.config import DispatcherConfig
    from DWDP.dispatcher.registry import build_dispatcher
    from DWDP.executor.registry import get_executor_class
    from DWDP.merger.config import MergerConfig
    from DWDP.merger.registry import build_merger
    from DWDP.router.config import RouterConfig
    from DWDP.router.registry import build_router
    from DWDP.scheduler.config import SchedulerConfig
    from DWDP.scheduler.registry import build_scheduler

    names = pkg.reference_plugin.register_with_reference()
    assert pkg.reference_plugin.register_with_reference() == names  # a second call is harmless
    r = build_router(RouterConfig(hidden_size=256, num_experts=8, top_k=2, router_type=names["router"]))
    assert isinstance(r, pkg.stages.B200LinearTopKRouter)
    d = build_dispatcher(DispatcherConfig(num_experts=8, dispatcher_type=names["dispatcher"], validate_inputs=False))
    assert isinstance(d, pkg.stages.B200ExpertMajorDispatcher)
    s = build_scheduler(SchedulerConfig(scheduling_policy=names["scheduler"]))
    assert isinstance(s, pkg.reference_plugin.ReferenceRoundRobinScheduler)
    m = build_merger(MergerConfig(backend=names["merger"]))
    assert isinstance(m, pkg.stages.B200Merger)
    assert get_executor_class(names["executor"]) is pkg.stages.B200Executor


def test_tensor_list_fields_follow_the_reference(pkg):
    from DWDP.executor.tensor_list import TensorList, _FIELD_NAMES

    assert tuple(pkg.tensor_list.FIELD_NAMES) == tuple(_FIELD_NAMES)
    ref = [f.name for f in dataclasses.fields(TensorList)]
    ours = [f.name for f in dataclasses.fields(pkg.tensor_list.TensorList)]
    assert ours[: len(ref)] == ref
    assert len(_FIELD_NAMES) + 1 == pkg._lib.TL_ROWS  # + the down-scale row


class _Mapping:
    def __init__(self, owner, size):
        self.owner_rank, self.size_bytes = owner, size


class _Table:
    def __init__(self, E, G, sizes):
        per = -(-E // G)
        self.m = {e: _Mapping(min(e // per, G - 1), sizes[e]) for e in range(E)}

    def get_mapping(self, e):
        return self.m[e]


class _Topo:
    def __init__(self, fn):
        self.fn = fn

    def canAccess(self, s, d):  # noqa: N802 - the reference's binding name
        return self.fn(s, d)


@pytest.mark.parametrize("E,G,rank,p2p", [(60, 4, 1, True), (60, 8, 5, False), (8, 2, 0, True), (256, 8, 7, True)])
def test_dwdp_planner_matches_the_reference_plan(pkg, E, G, rank, p2p):
    """Every descriptor, transfer, group, prefetch entry and statistic of the B200 planner's
    plan equals the reference's ExpertParallelPlanner (comms_planner/expert_parallel.py:182-359)
    on the same ownership, expert sizes and peer reachability."""
    from DWDP.comms_planner.config import CommunicationPlannerConfig as RefCfg
    from DWDP.comms_planner.expert_parallel import ExpertParallelPlanner

    sizes = [8_650_752 + (e % 3) * 1_000_003 for e in range(E)]  # ragged: last slices short
    access = (lambda s, d: True) if p2p else (lambda s, d: s == d)
    ref = ExpertParallelPlanner(RefCfg(planner_policy="expert_parallel", world_size=G, local_rank=rank,
                                       local_gpu_id=rank))
    ref.attach_expert_table(_Table(E, G, sizes))
    ref._peer_topology = _Topo(access)
    ref._scheduler = None
    ep = type("EP", (), {"expert_queue": torch.zeros(E, dtype=torch.int64)})()
    want = ref(ep)
    st = pkg.stages
    got = st.DWDPCommunicationPlanner(st.CommunicationPlannerConfig("expert_parallel", G, rank),
                                      bytes_per_expert=lambda e: sizes[e], peer_access=access)(ep)
    assert torch.equal(got.local_expert_ids, want.local_expert_ids)
    assert torch.equal(got.remote_expert_ids, want.remote_expert_ids)
    astuple = lambda d: tuple(getattr(d, f.name) for f in dataclasses.fields(d))  # noqa: E731
    assert [astuple(d) for d in got.communication_descriptors] == [astuple(d) for d in want.communication_descriptors]
    assert [astuple(d) for d in got.transfer_descriptors] == [astuple(d) for d in want.transfer_descriptors]
    assert len(got.communication_groups) == len(want.communication_groups)
    for a, b in zip(got.communication_groups, want.communication_groups):
        assert (a.group_id, a.source_gpu, a.destination_gpu) == (b.group_id, b.source_gpu, b.destination_gpu)
        assert torch.equal(a.descriptor_ids, b.descriptor_ids)
    assert torch.equal(got.prefetch.prefetch_expert_ids, want.prefetch.prefetch_expert_ids)
    assert torch.equal(got.prefetch.prefetch_priorities, want.prefetch.prefetch_priorities)
    assert astuple(got.statistics) == astuple(want.statistics)
    assert got.cost_model.total_estimated_bytes == want.cost_model.total_estimated_bytes
    assert torch.equal(got.topology.nvlink_connectivity, want.topology.nvlink_connectivity)
    assert got.topology.fabric == want.topology.fabric


@pytest.mark.parametrize("name", ["CommunicationPlan", "CommunicationDescriptor", "TransferDescriptor",
                                  "CommunicationGroup", "SynchronizationMetadata", "DependencyMetadata",
                                  "PrefetchPlan", "OverlapPlan", "CommunicationStatistics"])
def test_communication_plan_fields_cover_the_reference(pkg, name):
    import importlib

    ref = getattr(importlib.import_module("DWDP.comms_planner.metadata"), name)
    ours = getattr(pkg.comms_metadata, name)
    rf = [f.name for f in dataclasses.fields(ref)]
    assert [f.name for f in dataclasses.fields(ours)][: len(rf)] == rf

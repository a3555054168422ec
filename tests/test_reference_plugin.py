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

"""Plugging the B200 stages into the reference framework's own registries.

A deployment that keeps the reference (``DWDP``) as its host framework calls
:func:`register_with_reference` once; afterwards the reference's builders construct
the B200 stages by name, e.g. ``RuntimeConfig(dispatcher_type="b200_expert_major",
scheduling_policy="b200_round_robin", executor_backend="b200", merger_backend="b200")``
for ``DWDPRuntime.build_reference`` (DWDP/runtime/runtime.py:76-155).

Registered names (the reference's ``register_*`` functions, ``*/registry.py``):

================== ====================== ==============================================
registry           name                   class
================== ====================== ==============================================
router             ``b200_linear_topk``   :class:`stages.B200LinearTopKRouter`
dispatcher         ``b200_expert_major``  :class:`stages.B200ExpertMajorDispatcher`
scheduler          ``b200_round_robin``   :class:`ReferenceRoundRobinScheduler`
executor           ``b200``               :class:`stages.B200Executor`
merger             ``b200``               :class:`stages.B200Merger`
================== ====================== ==============================================

The stages take the reference's config objects (they read the same field names) and
return dataclasses with the reference's field sets (:mod:`plans`), so a reference stage
can consume a B200 stage's output and the other way round: the reference's PyTorch
merger merges the B200 executor's rows, the B200 executor runs the reference
scheduler's plan. Only the scheduler differs from its B200 form: the reference's
executors walk the plan's rows on the host and expect exactly the active experts, so
the registered scheduler returns the materialised (unpadded) plan.
"""
from __future__ import annotations

import importlib

from . import stages

REGISTERED = {
    "router": ("b200_linear_topk", "DWDP.router.registry", "register_router"),
    "dispatcher": ("b200_expert_major", "DWDP.dispatcher.registry", "register_dispatcher"),
    "scheduler": ("b200_round_robin", "DWDP.scheduler.registry", "register_scheduler"),
    "executor": ("b200", "DWDP.executor.registry", "register_executor"),
    "merger": ("b200", "DWDP.merger.registry", "register_merger"),
}


class ReferenceRoundRobinScheduler(stages.B200RoundRobinScheduler):
    """The B200 round-robin schedule in the reference's variable-length form (one row per
    active expert, DWDP/scheduler/policies/round_robin.py:23-89); reading the number of
    active experts back is the one host synchronisation, as in the reference."""

    def forward(self, dispatch_plan, workspace=None):
        return super().forward(dispatch_plan, workspace).materialize()


def _classes() -> dict[str, type]:
    return {"router": stages.B200LinearTopKRouter, "dispatcher": stages.B200ExpertMajorDispatcher,
            "scheduler": ReferenceRoundRobinScheduler, "executor": stages.B200Executor,
            "merger": stages.B200Merger}


def register_with_reference() -> dict[str, str]:
    """Register every B200 stage in the importable ``DWDP`` package's registries (idempotent:
    names already registered by an earlier call are left as they are). Returns kind -> name."""
    classes = _classes()
    done = {}
    for kind, (name, module, fn) in REGISTERED.items():
        mod = importlib.import_module(module)
        try:
            getattr(mod, fn)(name, classes[kind])
        except ValueError as exc:  # the reference refuses duplicate names
            if "already registered" not in str(exc):
                raise
        done[kind] = name
    return done

"""B200-native DWDP MoE-layer hot path.

The directory name is not a Python identifier; ``__graft_entry__.load_package()``
imports it as ``dwdp_b200``.
"""
from . import _lib, ops  # noqa: F401
from .weights import ExpertWeightStore  # noqa: F401
from .layer import MoELayer, algorithmic_bytes, algorithmic_flops  # noqa: F401

__all__ = ["_lib", "ops", "ExpertWeightStore", "MoELayer", "algorithmic_bytes", "algorithmic_flops"]
from . import comms_metadata, cost_model, decode, ep, hf_adapter, plans, reference_plugin, stages, tensor_list  # noqa: F401,E402
from .fused import fused_moe  # noqa: F401,E402

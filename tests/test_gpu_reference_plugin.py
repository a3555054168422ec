"""The B200 stages inside the reference's own runtime on the GPU: DWDPRuntime.build_reference
(DWDP/runtime/runtime.py:76-155) built by name from RuntimeConfig, with the B200 stages
mixed with the reference's (the reference merger merging the B200 executor's rows; the
B200 executor running the reference dispatcher's and scheduler's plans), against the CPU
oracle on the same dequantised weights and routing."""
from __future__ import annotations

import pytest
import torch

from tests.reference_import import import_reference

DWDP = import_reference()
pytestmark = [pytest.mark.gpu, pytest.mark.skipif(DWDP is None, reason="the reference package is not present")]
DEV = "cuda"
E, H, I, K = 8, 256, 384, 2

COMBOS = {
    "all_b200": dict(dispatcher_type="b200_expert_major", scheduling_policy="b200_round_robin",
                     executor_backend="b200", merger_backend="b200"),
    "reference_merger": dict(dispatcher_type="b200_expert_major", scheduling_policy="b200_round_robin",
                             executor_backend="b200", merger_backend="pytorch"),
    "reference_plans": dict(dispatcher_type="expert_major", scheduling_policy="round_robin",
                            executor_backend="b200", merger_backend="pytorch"),
}


class QwenExpert(torch.nn.Module):
    def __init__(self, g):
        super().__init__()
        self.gate_proj = torch.nn.Linear(H, I, bias=False)
        self.up_proj = torch.nn.Linear(H, I, bias=False)
        self.down_proj = torch.nn.Linear(I, H, bias=False)
        with torch.no_grad():
            for lin in (self.gate_proj, self.up_proj, self.down_proj):
                lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)

    def forward(self, x):
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


@pytest.mark.parametrize("combo", sorted(COMBOS))
def test_reference_runtime_with_b200_stages(pkg, orc, combo):
    from DWDP.router.config import MetadataLevel, RouterConfig
    from DWDP.router.registry import build_router
    from DWDP.runtime.config import RuntimeConfig
    from DWDP.runtime.runtime import DWDPRuntime

    pkg.reference_plugin.register_with_reference()
    g = torch.Generator().manual_seed(9)
    experts = [QwenExpert(g) for _ in range(E)]
    router = build_router(RouterConfig(hidden_size=H, num_experts=E, top_k=K, metadata_level=MetadataLevel.COUNTS))
    with torch.no_grad():
        router.weight.copy_(torch.randn(E, H, generator=g) / H**0.5)
    router = router.to(DEV, torch.bfloat16)
    cfg = RuntimeConfig(device="cuda", **COMBOS[combo])
    rt = DWDPRuntime.build_reference(hidden_size=H, num_experts=E, top_k=K, experts=experts, config=cfg,
                                     router=router)
    assert isinstance(rt.executor, pkg.stages.B200Executor)
    x = torch.randn(3, 41, H, generator=g).bfloat16()
    with torch.inference_mode():
        res = rt(x.to(DEV))
    y = res.merger_output.hidden_states
    torch.cuda.synchronize()
    assert y.shape == (3, 41, H)
    ro = res.router_output
    store = rt.executor.store
    deq = [tuple(t.cpu() for t in store.dequantized(e)) for e in range(E)]
    ref = orc.moe_forward(x.reshape(-1, H).float(), ro.topk_indices.reshape(-1, K).cpu(),
                          ro.topk_weights.reshape(-1, K).float().cpu(), deq)
    err = orc.rel_frobenius(y.reshape(-1, H).float().cpu(), ref)
    assert err < 2e-2, f"{combo}: rel Frobenius {err:.3e}"
    # the plans carry the reference's statistics fields, read on demand
    st = res.execution_plan.statistics
    assert st.num_experts == E and st.num_assignments == 3 * 41 * K

"""The reference-shaped stage operators and fused_moe on the GPU: the chained
stages must reproduce MoELayer bit for bit (same kernels), the plans must carry
the reference's integer values, and fused_moe must match the oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


class QwenExpert(torch.nn.Module):
    def __init__(self, H, I, g):
        super().__init__()
        self.gate_proj = torch.nn.Linear(H, I, bias=False)
        self.up_proj = torch.nn.Linear(H, I, bias=False)
        self.down_proj = torch.nn.Linear(I, H, bias=False)
        with torch.no_grad():
            for lin in (self.gate_proj, self.up_proj, self.down_proj):
                lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)


def test_stage_chain_matches_layer_and_oracle(pkg, orc):
    st = pkg.stages
    E, H, I, K, T = 8, 256, 384, 2, 77
    g = torch.Generator().manual_seed(5)
    experts = [QwenExpert(H, I, g) for _ in range(E)]
    rt = st.B200Runtime.build_reference(hidden_size=H, num_experts=E, top_k=K, experts=experts,
                                        executor_config=st.ExecutorConfig(weight_dtype=torch.bfloat16,
                                                                          scale_mode=pkg._lib.SCALE_NONE))
    rt.router.to(DEV)
    with torch.no_grad():
        rt.router.weight.copy_((torch.randn(E, H, generator=g) / H**0.5).bfloat16())
    x = torch.randn(3, T, H, generator=g).bfloat16().to(DEV)
    res = rt(x)
    assert res.hidden_states.shape == (3, T, H)
    ro, dp = res.router_output, res.dispatch_plan
    ref = orc.counting_scatter(ro.topk_indices.reshape(-1).cpu().numpy(), ro.topk_weights.reshape(-1).cpu().numpy(),
                               E, K)
    assert np.array_equal(dp.metadata.expert_offsets.cpu().numpy(), ref["offsets"])
    assert np.array_equal(dp.assignments.packed_token_indices.cpu().numpy(), ref["tok"])
    sched = orc.round_robin_schedule(ref["counts"], ref["offsets"])
    full = res.execution_plan.materialize()
    assert np.array_equal(full.expert_queue.cpu().numpy(), sched["expert_queue"])
    assert np.array_equal(full.expert_starts.cpu().numpy(), sched["expert_starts"])
    layer = pkg.MoELayer(rt.router.weight.detach(), rt.executor.store, K)
    assert torch.equal(layer(x), res.hidden_states)  # same kernels -> identical bits
    ex = [(m.gate_proj.weight.detach().bfloat16().float(), m.up_proj.weight.detach().bfloat16().float(),
           m.down_proj.weight.detach().bfloat16().float()) for m in experts]
    o = orc.moe_forward(x.reshape(-1, H).float().cpu(), ro.topk_indices.reshape(-1, K).cpu(),
                        ro.topk_weights.reshape(-1, K).cpu(), ex)
    assert orc.rel_frobenius(res.hidden_states.reshape(-1, H).float().cpu(), o) < 5e-3
    assert res.hidden_states.data_ptr() != res.executor_output.weighted_expert_outputs.data_ptr()


def test_executor_gathers_when_plan_has_no_rows(pkg, orc):
    st = pkg.stages
    E, H, I, K, T = 4, 128, 128, 2, 33
    g = torch.Generator().manual_seed(6)
    experts = [QwenExpert(H, I, g) for _ in range(E)]
    ex = st.B200Executor(st.ExecutorConfig(), experts)
    router = st.B200LinearTopKRouter(st.RouterConfig(H, E, K)).to(DEV)
    x = torch.randn(T, H, generator=g).bfloat16().to(DEV)
    ro = router(x)
    dp = st.B200ExpertMajorDispatcher(st.DispatcherConfig(E))(ro)  # no hidden: executor must gather
    assert dp.packed_hidden is None
    eo = ex(x, dp, st.B200RoundRobinScheduler(st.SchedulerConfig())(dp))
    y = st.B200Merger()(eo).hidden_states
    deq = [tuple(t.cpu() for t in ex.store.dequantized(e)) for e in range(E)]
    o = orc.moe_forward(x.float().cpu(), ro.topk_indices.cpu(), ro.topk_weights.cpu(), deq)
    assert orc.rel_frobenius(y.float().cpu(), o) < 2e-2


@pytest.mark.parametrize("layout", ["out_in", "in_out"])
def test_fused_moe_matches_oracle(pkg, orc, layout):
    E, H, I, K, T = 6, 384, 256, 2, 100
    g = torch.Generator().manual_seed(9)
    gate = torch.randn(E, I, H, generator=g) * 0.02
    up = torch.randn(E, I, H, generator=g) * 0.02
    down = torch.randn(E, H, I, generator=g) * 0.02
    if layout == "out_in":
        w1, w2 = torch.cat([gate, up], 1), down
    else:
        w1, w2 = torch.cat([gate, up], 1).transpose(1, 2).contiguous(), down.transpose(1, 2).contiguous()
    x = torch.randn(T, H, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g)
    w1d, w2d = w1.to(DEV), w2.to(DEV)
    y = pkg.fused_moe(x.to(DEV), w1d, w2d, ids.to(DEV), w.to(DEV))
    assert y.dtype == torch.bfloat16 and y.shape == (T, H)
    ex = [(gate[e].bfloat16().float(), up[e].bfloat16().float(), down[e].bfloat16().float()) for e in range(E)]
    ref = orc.moe_forward(x.float(), ids, w, ex)
    assert orc.rel_frobenius(y.float().cpu(), ref) < 5e-3
    y2 = pkg.fused_moe(x.to(DEV), w1d, w2d, ids.to(DEV), w.to(DEV))  # cached store
    assert torch.equal(y, y2)


def test_fused_moe_rejects_ambiguous_square(pkg):
    w1 = torch.zeros(2, 256, 256, device=DEV)
    w2 = torch.zeros(2, 256, 128, device=DEV)
    with pytest.raises(ValueError, match="ambiguous"):
        pkg.fused_moe(torch.zeros(4, 256, device=DEV), w1, w2, torch.zeros(4, 1, dtype=torch.long, device=DEV),
                      torch.ones(4, 1, device=DEV))

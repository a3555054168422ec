"""TensorList on the GPU: the device-built descriptor carries the plan's values in the
reference's fields (DWDP/executor/tensor_list.py:69-198), and the grouped GEMMs driven by
it (dwdp_grouped_moe) give the same bits as the per-expert launch and match the oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(pkg, E, H, I, K, T, seed, *, weight_dtype=torch.float8_e4m3fn, scale_mode=None, skip_expert=None):
    st = pkg.stages
    g = torch.Generator().manual_seed(seed)
    gate, up, down = (torch.randn(E, I, H, generator=g) * 0.02, torch.randn(E, I, H, generator=g) * 0.02,
                      torch.randn(E, H, I, generator=g) * 0.02)
    sm = scale_mode if scale_mode is not None else (pkg._lib.SCALE_CHANNEL if weight_dtype != torch.bfloat16
                                                    else pkg._lib.SCALE_NONE)
    store = pkg.ExpertWeightStore.from_weights(gate, up, down, weight_dtype=weight_dtype, scale_mode=sm, device=DEV)
    router = st.B200LinearTopKRouter(st.RouterConfig(H, E, K)).to(DEV)
    w = torch.randn(E, H, generator=g) / H**0.5
    with torch.no_grad():
        router.weight.copy_(w.bfloat16())
    x = torch.randn(T, H, generator=g).bfloat16().to(DEV)
    ro = router(x)
    if skip_expert is not None:  # route its slots to the next expert: it gets no rows
        ro.topk_indices.masked_fill_(ro.topk_indices == skip_expert, (skip_expert + 1) % E)
    dp = st.B200ExpertMajorDispatcher(st.DispatcherConfig(E))(ro)
    plan = st.B200RoundRobinScheduler(st.SchedulerConfig(stream_count=2))(dp)
    return store, x, ro, dp, plan


@pytest.mark.parametrize("materialized", [False, True])
def test_fields_follow_the_plan(pkg, materialized):
    tlm = pkg.tensor_list
    E, H, I, K, T = 16, 256, 384, 2, 50
    store, x, ro, dp, plan = _setup(pkg, E, H, I, K, T, 21, skip_expert=5)
    if materialized:
        plan = plan.materialize()  # the reference's variable-length plan
    weighted = torch.empty(T * K, H, dtype=torch.bfloat16, device=DEV)
    packed = torch.empty_like(weighted)
    inter = torch.empty(T * K, 2 * I, dtype=torch.bfloat16, device=DEV)
    ws = tlm.TensorListWorkspace(DEV)
    tl = tlm.TensorList.from_plans(x, dp, plan, ws, store, packed, weighted, inter)
    counts = dp.metadata.expert_counts.cpu().numpy()
    offsets = dp.metadata.expert_offsets.cpu().numpy()
    active = np.nonzero(counts > 0)[0]
    assert 5 not in active and tl.size == len(active)
    assert tl.launch_dimensions == (int(counts.max()), H, 2 * I)
    f = {n: getattr(tl, n).cpu().numpy() for n in tlm.FIELD_NAMES}
    assert np.array_equal(f["expert_ids"], active)
    assert np.array_equal(f["token_offsets"], offsets[active])
    assert np.array_equal(f["token_counts"], counts[active]) and np.array_equal(f["m"], counts[active])
    w13 = store.w13_ptrs.cpu().numpy()
    assert np.array_equal(f["gate_weight_ptrs"], w13[active]) and np.array_equal(f["up_weight_ptrs"], w13[active])
    assert np.array_equal(f["down_weight_ptrs"], store.w2_ptrs.cpu().numpy()[active])
    assert np.array_equal(f["quantization_ptrs"], store.s13_ptrs.cpu().numpy()[active])
    assert np.array_equal(tl.down_quantization_ptrs.cpu().numpy(), store.s2_ptrs.cpu().numpy()[active])
    rb = H * 2
    assert np.array_equal(f["weighted_output_ptrs"], weighted.data_ptr() + offsets[active] * rb)
    assert np.array_equal(f["output_ptrs"], packed.data_ptr() + offsets[active] * rb)
    assert np.array_equal(f["intermediate_ptrs"], inter.data_ptr() + offsets[active] * 4 * I)
    assert (f["input_ptrs"] == x.data_ptr()).all()
    assert (f["token_index_ptrs"] == dp.assignments.packed_token_indices.data_ptr()).all()
    assert (f["routing_weight_ptrs"] == dp.assignments.packed_routing_weights.data_ptr()).all()
    assert (f["n"] == H).all() and (f["k"] == H).all() and (f["intermediate_n"] == 2 * I).all()
    assert (f["input_ld"] == H).all() and (f["gate_ld"] == H).all() and (f["down_ld"] == I).all()
    assert (f["dtype_codes"] == 2).all()  # the reference's code for bf16
    assert np.array_equal(f["workspace_indices"], np.arange(len(active)))
    assert np.array_equal(f["execution_priorities"], np.arange(len(active)))
    assert np.array_equal(f["stream_ids"], np.arange(len(active)) % 2)
    # entries past the active count read as empty experts
    rest = ws.fields[:, tl.size:].cpu().numpy()
    if rest.size:
        assert (rest[10] == -1).all() and (np.delete(rest, 10, axis=0) == 0).all()


@pytest.mark.parametrize("cfg", [
    dict(E=60, H=2048, I=1408, K=4, T=64, wd=torch.float8_e4m3fn, sm="CHANNEL"),
    dict(E=60, H=2048, I=1408, K=4, T=700, wd=torch.float8_e4m3fn, sm="CHANNEL"),
    dict(E=8, H=512, I=384, K=2, T=200, wd=torch.float8_e4m3fn, sm="BLOCK128"),
    dict(E=8, H=256, I=256, K=2, T=33, wd=torch.bfloat16, sm="NONE"),
])
def test_grouped_moe_from_tensor_list(pkg, orc, cfg):
    tlm = pkg.tensor_list
    E, H, I, K, T = cfg["E"], cfg["H"], cfg["I"], cfg["K"], cfg["T"]
    sm = getattr(pkg._lib, "SCALE_" + cfg["sm"])
    store, x, ro, dp, plan = _setup(pkg, E, H, I, K, T, 31, weight_dtype=cfg["wd"], scale_mode=sm)
    md = dp.metadata
    N = T * K
    status = torch.zeros(4, dtype=torch.int32, device=DEV)
    # the per-expert launch
    ref_out = torch.empty(N, H, dtype=torch.bfloat16, device=DEV)
    ws = torch.empty(pkg.ops.moe_workspace_bytes(T, K, E, I, 0), dtype=torch.uint8, device=DEV)
    w = dp.assignments.packed_routing_weights.float()
    pkg.ops.moe_experts(store.group(), None, None, x, K, md.expert_counts, md.expert_offsets, w, None, ref_out,
                        None, ws, status, packed_token_indices=dp.assignments.packed_token_indices)
    # the same GEMMs driven by the TensorList, twice (the second reuses the workspace)
    tws = tlm.TensorListWorkspace(DEV)
    for sync in (True, False):
        out = torch.full((N, H), float("nan"), dtype=torch.bfloat16, device=DEV)
        tl = tlm.TensorList.from_plans(x, dp, plan, tws, store, None, out, None, sync=sync)
        mws = torch.empty(pkg.ops.moe_workspace_bytes(T, K, tl.capacity, I, 0), dtype=torch.uint8, device=DEV)
        tlm.grouped_moe(tl, x, dp, out, mws, status=status)
        torch.cuda.synchronize()
        assert status[0].item() == 0, status.tolist()
        assert torch.equal(out, ref_out)
    deq = [tuple(t.cpu() for t in store.dequantized(e)) for e in range(E)]
    o = orc.moe_forward(x.float().cpu(), ro.topk_indices.cpu(), ro.topk_weights.cpu(), deq)
    y = torch.zeros(T, H)
    y.index_add_(0, dp.assignments.packed_token_indices.cpu(), out.float().cpu())
    tol = 5e-3 if cfg["wd"] == torch.bfloat16 else 2e-2
    assert orc.rel_frobenius(y, o) < tol


def test_executor_on_tensor_list_matches_default(pkg):
    st = pkg.stages
    E, H, I, K, T = 12, 512, 256, 2, 90
    store, x, ro, dp, plan = _setup(pkg, E, H, I, K, T, 41)
    a = st.B200Executor(st.ExecutorConfig(), store)(x, dp, plan)
    b = st.B200Executor(st.ExecutorConfig(use_tensor_list=True), store)(x, dp, plan)
    assert torch.equal(a.weighted_expert_outputs, b.weighted_expert_outputs)


def test_capacity_and_contract_errors(pkg):
    tlm = pkg.tensor_list
    E, H, I, K, T = 8, 256, 256, 2, 16
    store, x, ro, dp, plan = _setup(pkg, E, H, I, K, T, 51)
    with pytest.raises(ValueError):
        tlm.TensorListWorkspace(DEV).ensure_capacity(2048)
    with pytest.raises(ValueError):
        tlm.TensorList.from_plans(x[:, :128], dp, plan, tlm.TensorListWorkspace(DEV), store, None, None, None)
    w1 = torch.empty(T * K, H, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        tlm.TensorList.from_plans(x, dp, plan, tlm.TensorListWorkspace(DEV), store, w1[:, :8], w1, None)

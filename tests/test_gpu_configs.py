"""MoE-layer parity at the other BASELINE shapes: Mixtral-8x7B (H 4096, 8 experts,
FFN 14336, top-2, 128x128 block scales, Zipf-skewed routing) and DeepSeek-V3
(H 7168, 256 experts, FFN 2048, top-8, one shared expert, block scales).

Weights are generated one expert at a time on the GPU (the DeepSeek shape's
256 fp32 experts would need ~45 GB of host memory) and only the experts a batch
activates are dequantised for the fp32 CPU oracle."""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
FP8_TOL = 2e-2


def _store(pkg, E, H, I, seed):
    st = pkg.ExpertWeightStore(E, H, I, weight_dtype=torch.float8_e4m3fn, scale_mode=pkg._lib.SCALE_BLOCK128,
                               device=DEV)
    g = torch.Generator(device=DEV).manual_seed(seed)
    for e in range(E):
        gate = torch.randn(I, H, generator=g, device=DEV) * 0.02
        up = torch.randn(I, H, generator=g, device=DEV) * 0.02
        down = torch.randn(H, I, generator=g, device=DEV) * 0.02
        st.load_expert(e, gate, up, down)
    return st


def _check(pkg, orc, layer, x, tol=FP8_TOL):
    T = x.shape[0]
    y = layer(x.to(DEV))
    torch.cuda.synchronize()
    assert layer.read_status(T)[0] == 0
    ws = layer.workspace(T)
    idx, wts = ws.router.topk_indices.cpu(), ws.router.topk_weights.cpu()
    active = sorted(set(idx.reshape(-1).tolist()))
    experts = [None] * layer.num_experts
    for e in active:
        experts[e] = tuple(t.cpu() for t in layer.experts.dequantized(e))
    shared = tuple(t.cpu() for t in layer.shared_expert.dequantized(0)) if layer.shared_expert else None
    sgate = ws.router.shared_gate.cpu() if ws.router.shared_gate is not None else None
    ref = orc.moe_forward(x.float(), idx, wts, experts, shared=shared, shared_gate=sgate)
    err = orc.rel_frobenius(y.float().cpu(), ref)
    assert err < tol, f"rel Frobenius {err:.3e}"
    return err, active


def test_mixtral_shape_zipf_routing(pkg, orc):
    E, H, I, K = 8, 4096, 14336, 2
    g = torch.Generator().manual_seed(1236)
    router = (torch.randn(E, H, generator=g) / math.sqrt(H)).bfloat16()
    rank = torch.randperm(E, generator=g)
    bias = (-1.2 * torch.log(rank.float() + 1.0)).float()  # Zipf(s=1.2)-shaped expert loads
    layer = pkg.MoELayer(router.to(DEV), _store(pkg, E, H, I, 1236), K, router_bias=bias.to(DEV))
    # the load histogram falls off with the expert's rank
    xs = torch.randn(8192, H, generator=g).bfloat16().to(DEV)
    res = pkg.ops.router_topk(xs, layer.router_weight, K, bias=layer.router_bias)
    load = torch.bincount(res.topk_indices.reshape(-1).cpu(), minlength=E).float()
    by_rank = load[torch.argsort(rank)]
    lr = torch.log(torch.arange(1, E + 1).float())
    ll = torch.log(by_rank.clamp_min(1.0))
    fit = ((lr - lr.mean()) * (ll - ll.mean())).sum() / ((lr - lr.mean()) ** 2).sum()
    assert fit < -0.5, f"log-log load slope {fit:.2f} is not Zipf-like"
    for T in (1, 16):
        x = torch.randn(T, H, generator=g).bfloat16()
        _check(pkg, orc, layer, x)


def test_deepseek_shape_block_scales(pkg, orc):
    E, H, I, K, Is = 256, 7168, 2048, 8, 2048
    g = torch.Generator().manual_seed(1237)
    router = (torch.randn(E, H, generator=g) / math.sqrt(H)).bfloat16()
    gate_w = (torch.randn(H, generator=g) * 0.02).bfloat16()
    layer = pkg.MoELayer(router.to(DEV), _store(pkg, E, H, I, 1237), K,
                         shared_expert=_store(pkg, 1, H, Is, 1238), shared_gate_weight=gate_w.to(DEV))
    x = torch.randn(2, H, generator=g).bfloat16()
    _, active = _check(pkg, orc, layer, x)
    assert len(active) >= 8

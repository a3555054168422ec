"""Parity at the sizes bench.py measures, against the CPU oracle.

* the Qwen-shaped layer at T = 4096 (the headline point) in both activation modes;
* the 4-layer chain exactly as bench.py builds and runs it (LayerStack), the oracle
  chained through the same seeded layers with each layer's GPU routing;
* Mixtral-8x7B at a prefill size (T = 512, 128x128 block scales, Zipf-skewed routing)
  and DeepSeek-V3 at T = 256.

Experts are dequantised one at a time, only when the routing selects them, so the
DeepSeek shape (256 experts of 3 x 7168 x 2048) never needs all of them in host memory."""
from __future__ import annotations

import math

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu
DEV = "cuda"
FP8_TOL = 2e-2


class LazyExperts:
    """Indexable over a store's experts: item e is expert e dequantised to fp32 on the CPU."""

    def __init__(self, store):
        self.store = store

    def __len__(self):
        return self.store.num_experts

    def __getitem__(self, e):
        return tuple(t.cpu() for t in self.store.dequantized(e))


def oracle_act(layer) -> str:
    return "block128" if layer.activation_quant == "block128" else "none"


def oracle_layer(orc, layer, x: torch.Tensor) -> torch.Tensor:
    """The oracle of ``layer`` on input ``x`` (fp32 CPU) with the routing of the layer's last
    GPU forward over the same number of tokens."""
    ws = layer.workspace(x.shape[0])
    shared = tuple(t.cpu() for t in layer.shared_expert.dequantized(0)) if layer.shared_expert else None
    sgate = ws.router.shared_gate.cpu() if ws.router.shared_gate is not None else None
    return orc.moe_forward(x, ws.router.topk_indices.cpu(), ws.router.topk_weights.cpu(), LazyExperts(layer.experts),
                           shared=shared, shared_gate=sgate, act_quant=oracle_act(layer))


@pytest.mark.parametrize("act", ["block128", "hilo"])
def test_qwen_layer_T4096(pkg, orc, act):
    layer = bench.make_qwen_layer(pkg, DEV, activation_quant=act)
    x = bench.make_inputs(4096, DEV, seed=4242)
    y = layer(x)
    torch.cuda.synchronize()
    assert layer.read_status(4096)[0] == 0
    err = orc.rel_frobenius(y.float().cpu(), oracle_layer(orc, layer, x.float().cpu()))
    assert err < FP8_TOL, f"{act}: rel Frobenius {err:.3e}"


def test_bench_layer_chain(pkg, orc):
    """bench.py's timed step: L = 4 chained layers at T = 4096, bench's activation mode. Every
    layer is checked against the oracle on the input the GPU chain actually gave it (with the
    routing the GPU computed). The chained oracle is not the bar: the synthetic layers have no
    residual path and shrink the signal ~50 000x over four layers, which amplifies any input
    difference, so the end-to-end error of two independently rounded chains measures that
    conditioning, not the kernels."""
    stack = bench.LayerStack(pkg, torch.device(DEV), 4, 4096, 0, 1)
    y = stack.step()
    torch.cuda.synchronize()
    x = stack.x0
    for l, lay in enumerate(stack.layers):
        assert lay.read_status(4096)[0] == 0
        out = stack.outs[l % 2] if l < len(stack.layers) - 1 else y
        if l < len(stack.layers) - 1:  # the buffer is rewritten two layers later: re-run this layer alone
            out = lay(x)
            torch.cuda.synchronize()
        err = orc.rel_frobenius(out.float().cpu(), oracle_layer(orc, lay, x.float().cpu()))
        assert err < FP8_TOL, f"layer {l} of the chain: rel Frobenius {err:.3e}"
        x = out


def _block_store(pkg, E, H, I, seed, act):
    st = pkg.ExpertWeightStore(E, H, I, weight_dtype=torch.float8_e4m3fn, scale_mode=pkg._lib.SCALE_BLOCK128,
                               device=DEV, activation_quant=act)
    g = torch.Generator(device=DEV).manual_seed(seed)
    for e in range(E):
        st.load_expert(e, torch.randn(I, H, generator=g, device=DEV) * 0.02,
                       torch.randn(I, H, generator=g, device=DEV) * 0.02,
                       torch.randn(H, I, generator=g, device=DEV) * 0.02)
    return st


@pytest.mark.parametrize("act", ["block128", "hilo"])
def test_mixtral_prefill_T512(pkg, orc, act):
    E, H, I, K = 8, 4096, 14336, 2
    g = torch.Generator().manual_seed(1236)
    router = (torch.randn(E, H, generator=g) / math.sqrt(H)).bfloat16()
    rank = torch.randperm(E, generator=g)
    bias = (-1.2 * torch.log(rank.float() + 1.0)).float()  # Zipf(s=1.2)-shaped expert loads
    layer = pkg.MoELayer(router.to(DEV), _block_store(pkg, E, H, I, 1236, act), K, router_bias=bias.to(DEV))
    x = torch.randn(512, H, generator=g).bfloat16()
    y = layer(x.to(DEV))
    torch.cuda.synchronize()
    assert layer.read_status(512)[0] == 0
    err = orc.rel_frobenius(y.float().cpu(), oracle_layer(orc, layer, x.float()))
    assert err < FP8_TOL, f"{act}: rel Frobenius {err:.3e}"


def test_deepseek_T256(pkg, orc):
    E, H, I, K, Is = 256, 7168, 2048, 8, 2048
    g = torch.Generator().manual_seed(1237)
    router = (torch.randn(E, H, generator=g) / math.sqrt(H)).bfloat16()
    gate_w = (torch.randn(H, generator=g) * 0.02).bfloat16()
    layer = pkg.MoELayer(router.to(DEV), _block_store(pkg, E, H, I, 1237, "block128"), K,
                         shared_expert=_block_store(pkg, 1, H, Is, 1238, "block128"),
                         shared_gate_weight=gate_w.to(DEV))
    x = torch.randn(256, H, generator=g).bfloat16()
    y = layer(x.to(DEV))
    torch.cuda.synchronize()
    assert layer.read_status(256)[0] == 0
    err = orc.rel_frobenius(y.float().cpu(), oracle_layer(orc, layer, x.float()))
    assert err < FP8_TOL, f"rel Frobenius {err:.3e}"

"""Generate the golden fixtures in this directory by running the REFERENCE itself.

Run in a container where the reference project is importable:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own Python package (``DWDP``) and records, with
fixed seeds:

* ``dispatch_cases.npz``   counting_scatter_expert_major_dispatch outputs for the
  (T, E, K) grid of DWDP/tests/dispatcher/test_triton_dispatcher.py:68-109;
* ``router_cases.npz``     reference_topk_routing on fp32 logits;
* ``quant_cases.npz``      quantize_weights_blockwise / quantize_activations_blockwise;
* ``c1_pipeline.npz``      BASELINE config 1 (T256 H512 E8 K2 I1024, fp32) through
  DWDPRuntime.build_reference with Qwen-style SwiGLU experts: routing, dispatch
  plan and the final hidden states.

Inputs are regenerated from the seeds by :func:`c1_inputs` / :func:`dispatch_inputs`
(torch CPU generators), so the fixtures hold only outputs.
"""
from __future__ import annotations

import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent

DISPATCH_GRID = [(1, 1, 1), (8, 4, 1), (33, 8, 2), (127, 16, 4), (513, 8, 2), (513, 16, 4),
                 (1025, 64, 8), (2049, 128, 2)]
C1 = dict(T=256, H=512, E=8, K=2, I=1024, seed=1234)


def dispatch_inputs(T: int, E: int, K: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(1234 + T + E + K)
    ids = torch.randint(0, E, (T, K), generator=g, dtype=torch.int64)
    w = torch.rand(T, K, generator=g, dtype=torch.float32)
    return ids, w


def router_inputs(T: int, E: int, seed: int) -> torch.Tensor:
    return torch.randn(T, E, generator=torch.Generator().manual_seed(seed), dtype=torch.float32)


def c1_inputs() -> dict[str, torch.Tensor]:
    """x~N(0,1)[256,512]; router W~N(0,0.02)[8,512];
    gate_up [8,2048,512] and down [8,512,1024] ~N(0,0.02)."""
    g = torch.Generator().manual_seed(C1["seed"])
    T, H, E, I = C1["T"], C1["H"], C1["E"], C1["I"]
    x = torch.randn(T, H, generator=g)
    router_w = torch.randn(E, H, generator=g) * 0.02
    gate_up = torch.randn(E, 2 * I, H, generator=g) * 0.02
    down = torch.randn(E, H, I, generator=g) * 0.02
    return {"x": x, "router_w": router_w, "gate": gate_up[:, :I].contiguous(),
            "up": gate_up[:, I:].contiguous(), "down": down}


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    from DWDP.dispatcher.kernels.reference import counting_scatter_expert_major_dispatch
    from DWDP.executor.fp8 import quantize_activations_blockwise, quantize_weights_blockwise
    from DWDP.router.config import MetadataLevel, RouterConfig
    from DWDP.router.kernels.fused import reference_topk_routing
    from DWDP.router.registry import build_router
    from DWDP.runtime.runtime import DWDPRuntime

    # ---------------- dispatch
    out = {}
    for T, E, K in DISPATCH_GRID:
        ids, w = dispatch_inputs(T, E, K)
        r = counting_scatter_expert_major_dispatch(ids.reshape(-1), w.reshape(-1), num_experts=E, top_k=K)
        names = ["counts", "offsets", "perm", "inv", "ids", "tok", "weights"]
        for n, t in zip(names, r):
            out[f"{T}_{E}_{K}_{n}"] = t.numpy()
    np.savez_compressed(HERE / "dispatch_cases.npz", **out)

    # ---------------- router
    out = {}
    for T, E, K, seed in [(64, 60, 4, 1), (33, 8, 2, 2), (16, 256, 8, 3), (5, 4, 1, 4)]:
        logits = router_inputs(T, E, seed)
        for renorm in (True, False):
            p, i, w = reference_topk_routing(logits, K, renormalize=renorm)
            key = f"{T}_{E}_{K}_{seed}_{int(renorm)}"
            out[key + "_probs"] = p.numpy()
            out[key + "_idx"] = i.numpy()
            out[key + "_weights"] = w.numpy()
    np.savez_compressed(HERE / "router_cases.npz", **out)

    # ---------------- quantisation
    g = torch.Generator().manual_seed(5)
    wmat = torch.randn(384, 256, generator=g) * 0.02
    wmat[7, 3] = 1.5  # one hot block
    q, s = quantize_weights_blockwise(wmat, torch.float8_e4m3fn)
    act = torch.randn(9, 384, generator=g)
    aq, asc = quantize_activations_blockwise(act, torch.float8_e4m3fn)
    np.savez_compressed(HERE / "quant_cases.npz", w_q=q.view(torch.uint8).numpy(), w_s=s.numpy(),
                        a_q=aq.view(torch.uint8).numpy(), a_s=asc.numpy())

    # ---------------- BASELINE config 1 through the reference runtime
    inp = c1_inputs()
    T, H, E, K, I = C1["T"], C1["H"], C1["E"], C1["K"], C1["I"]

    class QwenSwiGLUExpert(torch.nn.Module):
        def __init__(self, gate, up, down):
            super().__init__()
            self.gate_proj = torch.nn.Linear(H, I, bias=False)
            self.up_proj = torch.nn.Linear(H, I, bias=False)
            self.down_proj = torch.nn.Linear(I, H, bias=False)
            with torch.no_grad():
                self.gate_proj.weight.copy_(gate)
                self.up_proj.weight.copy_(up)
                self.down_proj.weight.copy_(down)

        def forward(self, x):
            return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))

    experts = [QwenSwiGLUExpert(inp["gate"][e], inp["up"][e], inp["down"][e]) for e in range(E)]
    router = build_router(RouterConfig(hidden_size=H, num_experts=E, top_k=K, metadata_level=MetadataLevel.COUNTS))
    with torch.no_grad():
        router.weight.copy_(inp["router_w"])
    rt = DWDPRuntime.build_reference(hidden_size=H, num_experts=E, top_k=K, experts=experts, router=router)
    with torch.inference_mode():
        res = rt(inp["x"])
    ro = res.router_output
    md = res.dispatch_plan.metadata
    np.savez_compressed(
        HERE / "c1_pipeline.npz",
        hidden=res.hidden_states.numpy(),
        logits=ro.router_logits.numpy(),
        topk_idx=ro.topk_indices.numpy(),
        topk_weights=ro.topk_weights.numpy(),
        counts=md.expert_counts.numpy(),
        offsets=md.expert_offsets.numpy(),
        perm=md.token_permutation.numpy(),
        tok=res.dispatch_plan.assignments.packed_token_indices.numpy(),
    )
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")

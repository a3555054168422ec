"""Generate ``decode_attention.npz`` by running transformers' Qwen2-MoE attention
modules, the third-party code the reference's HF adapter keeps around its MoE
blocks (``DWDP/adapters/qwen15_moe.py:526-543``).

    python tests/golden/make_decode_golden.py

Needs only ``transformers`` (5.5 in this image). For each case, with fixed seeds,
it builds ``Qwen2MoeRMSNorm`` + ``Qwen2MoeRotaryEmbedding`` (rope_type default) +
``Qwen2MoeAttention`` (eager) in fp32 and runs a causal pass over L rows: the last
row's attention output is what a decode step at position L-1 computes against a
cache holding rows 0..L-2. Inputs and weights are regenerated from the seeds by
:func:`decode_case_inputs` (torch CPU generator), so the fixture holds only outputs.
"""
from __future__ import annotations

import pathlib

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent

# (hidden, heads, rows L, rope theta)
DECODE_CASES = [(256, 2, 1, 1e6), (256, 2, 37, 1e6), (512, 4, 130, 1e4)]
EPS = 1e-6


def decode_case_inputs(H: int, NH: int, L: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(L, H, generator=g)
    ln = 1.0 + 0.1 * torch.randn(H, generator=g)
    wqkv = torch.randn(3 * H, H, generator=g) / H**0.5
    bqkv = 0.1 * torch.randn(3 * H, generator=g)
    wo = torch.randn(H, H, generator=g) / H**0.5
    return x, ln, wqkv, bqkv, wo


def case_seed(i: int) -> int:
    return 2024 + i


def _hf_case(H, NH, L, theta, seed):
    from transformers import Qwen2MoeConfig
    from transformers.models.qwen2_moe import modeling_qwen2_moe as m

    cfg = Qwen2MoeConfig(hidden_size=H, num_attention_heads=NH, num_key_value_heads=NH, rms_norm_eps=EPS,
                         rope_parameters={"rope_type": "default", "rope_theta": theta},
                         max_position_embeddings=4096, attention_dropout=0.0)
    cfg._attn_implementation = "eager"
    x, ln, wqkv, bqkv, wo = decode_case_inputs(H, NH, L, seed)
    norm = m.Qwen2MoeRMSNorm(H, eps=EPS)
    norm.weight.data.copy_(ln)
    attn = m.Qwen2MoeAttention(cfg, layer_idx=0).eval()
    wq, wk, wv = wqkv.split(H)
    bq, bk, bv = bqkv.split(H)
    attn.q_proj.weight.data.copy_(wq)
    attn.k_proj.weight.data.copy_(wk)
    attn.v_proj.weight.data.copy_(wv)
    attn.q_proj.bias.data.copy_(bq)
    attn.k_proj.bias.data.copy_(bk)
    attn.v_proj.bias.data.copy_(bv)
    attn.o_proj.weight.data.copy_(wo)
    rot = m.Qwen2MoeRotaryEmbedding(cfg)
    with torch.no_grad():
        xn = norm(x[None])
        pos = torch.arange(L)[None]
        cos, sin = rot(xn, pos)
        mask = torch.full((L, L), float("-inf")).triu(1)[None, None]
        out, _ = attn(xn, position_embeddings=(cos, sin), attention_mask=mask)
    return xn[0].numpy(), out[0, -1].numpy()


def main() -> None:
    arrays = {}
    for i, (H, NH, L, theta) in enumerate(DECODE_CASES):
        xn, o = _hf_case(H, NH, L, theta, case_seed(i))
        arrays[f"c{i}_normed_last"] = xn[-1].astype(np.float32)
        arrays[f"c{i}_attn_last"] = o.astype(np.float32)
    np.savez_compressed(HERE / "decode_attention.npz", **arrays)
    print("wrote", HERE / "decode_attention.npz", {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()

"""CPU oracle of the model around the MoE layers in a Qwen1.5-MoE decode step: TEST
INFRASTRUCTURE ONLY. Only tests/, ``__graft_entry__.smoke()`` and bench.py's
``cpu_baseline`` leg use this module, as the checker; the product path never does.

The reference runs these parts through Hugging Face's Qwen2-MoE decoder layer
(``DWDP/adapters/qwen15_moe.py:526-543`` patches only the MoE block and keeps the
HF attention; the paged cache layout is ``DWDP/runtime/paged_attention.py:20-76``).
The third-party code is transformers' ``models/qwen2_moe/modeling_qwen2_moe.py``
(transformers 5.5 in this image: ``Qwen2MoeRMSNorm``, ``Qwen2MoeRotaryEmbedding``
with ``rope_type="default"``, ``apply_rotary_pos_emb``, ``Qwen2MoeAttention`` with
q/k/v bias and no o_proj bias, eager softmax attention). This file restates that
published algorithm in fp32 torch on the CPU; it is pinned against transformers'
own modules by ``tests/golden/make_decode_golden.py`` (fixture
``tests/golden/decode_attention.npz``).
"""
from __future__ import annotations

import math

import torch


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen2MoeRMSNorm: x * rsqrt(mean(x^2) + eps) * weight, in fp32."""
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight.float()


def rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half rotary embedding ([..., S, D] with positions [S]):
    inv_freq_d = theta^(-2d/D) for d < D/2, angle = pos * inv_freq repeated over both
    halves, out = x * cos + rotate_half(x) * sin with rotate_half(x) = [-x2, x1]."""
    D = x.shape[-1]
    inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = positions.double()[:, None] * inv_freq[None, :]
    emb = torch.cat([ang, ang], dim=-1)
    cos, sin = emb.cos().float(), emb.sin().float()
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    return x.float() * cos + torch.cat([-x2, x1], dim=-1).float() * sin


def attention_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """One query per head over a dense history: q [NH, D], k/v [L, NH, D] -> [NH, D]."""
    s = torch.einsum("hd,lhd->hl", q.float(), k.float()) * scale
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hl,lhd->hd", p, v.float())


def attention_block(x_hist: torch.Tensor, positions: torch.Tensor, wqkv: torch.Tensor, bqkv: torch.Tensor,
                    wo: torch.Tensor, num_heads: int, theta: float) -> torch.Tensor:
    """Attention output (after o_proj) for the LAST row of x_hist [L, H] (already normed),
    with every row's k/v projected and rotated at its position: the decode step of
    Qwen2MoeAttention with a cache holding rows 0..L-2."""
    L, H = x_hist.shape
    D = H // num_heads
    qkv = x_hist.float() @ wqkv.float().t() + bqkv.float()
    q, k, v = qkv.view(L, 3, num_heads, D).unbind(1)
    qr = rope(q.transpose(0, 1), positions, theta).transpose(0, 1)  # [L, NH, D]
    kr = rope(k.transpose(0, 1), positions, theta).transpose(0, 1)
    o = attention_decode(qr[-1], kr, v, 1.0 / math.sqrt(D))
    return o.reshape(H) @ wo.float().t()


def decoder_attention_half(h: torch.Tensor, ln_w: torch.Tensor, eps: float, k_hist: torch.Tensor,
                           v_hist: torch.Tensor, position: int, wqkv: torch.Tensor, bqkv: torch.Tensor,
                           wo: torch.Tensor, num_heads: int, theta: float):
    """First half of a decode-step decoder layer for one token against a cache that already
    holds (rotated) k_hist/v_hist [position, NH, D]: returns (attention output [H],
    k_new [NH, D] (rotated), v_new [NH, D])."""
    H = h.shape[-1]
    D = H // num_heads
    xn = rms_norm(h, ln_w, eps)
    qkv = xn @ wqkv.float().t() + bqkv.float()
    q, k, v = qkv.view(3, num_heads, D).unbind(0)
    pos = torch.tensor([position])
    qr = rope(q[:, None, :], pos, theta)[:, 0]
    kr = rope(k[:, None, :], pos, theta)[:, 0]
    keys = torch.cat([k_hist.float(), kr[None]], 0)
    vals = torch.cat([v_hist.float(), v[None]], 0)
    o = attention_decode(qr, keys, vals, 1.0 / math.sqrt(D))
    return o.reshape(H) @ wo.float().t(), kr, v

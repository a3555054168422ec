"""Pin the decode-step oracle (oracle/decode_oracle.py) against transformers'
Qwen2-MoE RMSNorm / rotary / attention modules (fixture made by
tests/golden/make_decode_golden.py), plus size-independent properties."""
from __future__ import annotations

import math
import pathlib

import numpy as np
import pytest
import torch

from oracle import decode_oracle as dor
from tests.golden.make_decode_golden import DECODE_CASES, EPS, case_seed, decode_case_inputs

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "decode_attention.npz"


@pytest.mark.parametrize("i", range(len(DECODE_CASES)))
def test_oracle_matches_transformers(i):
    H, NH, L, theta = DECODE_CASES[i]
    gold = np.load(GOLDEN)
    x, ln, wqkv, bqkv, wo = decode_case_inputs(H, NH, L, case_seed(i))
    xn = dor.rms_norm(x, ln, EPS)
    np.testing.assert_allclose(xn[-1].numpy(), gold[f"c{i}_normed_last"], rtol=1e-5, atol=1e-5)
    o = dor.attention_block(xn, torch.arange(L), wqkv, bqkv, wo, NH, theta)
    np.testing.assert_allclose(o.numpy(), gold[f"c{i}_attn_last"], rtol=1e-4, atol=1e-4)


def test_incremental_half_matches_full_block():
    """decoder_attention_half against a cache built row by row equals the causal block."""
    H, NH, L, theta = 256, 2, 9, 1e6
    x, ln, wqkv, bqkv, wo = decode_case_inputs(H, NH, L, 77)
    D = H // NH
    ks, vs = torch.zeros(0, NH, D), torch.zeros(0, NH, D)
    for p in range(L):
        o, k, v = dor.decoder_attention_half(x[p], ln, EPS, ks, vs, p, wqkv, bqkv, wo, NH, theta)
        ks, vs = torch.cat([ks, k[None]]), torch.cat([vs, v[None]])
    full = dor.attention_block(dor.rms_norm(x, ln, EPS), torch.arange(L), wqkv, bqkv, wo, NH, theta)
    torch.testing.assert_close(o, full, rtol=1e-5, atol=1e-5)


def test_rope_preserves_norm_and_relative_angle():
    g = torch.Generator().manual_seed(5)
    q, k = torch.randn(1, 128, generator=g), torch.randn(1, 128, generator=g)
    for a, b in ((3, 1), (103, 101)):
        qa, kb = dor.rope(q, torch.tensor([a]), 1e6), dor.rope(k, torch.tensor([b]), 1e6)
        assert math.isclose(qa.norm().item(), q.norm().item(), rel_tol=1e-5)
        if a == 3:
            d0 = (qa * kb).sum().item()
        else:
            assert math.isclose((qa * kb).sum().item(), d0, rel_tol=1e-4, abs_tol=1e-4)

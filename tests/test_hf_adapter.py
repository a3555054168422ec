"""HF adapter host logic on CPU (discovery, patch/restore, routing mode, fp8 import
maths), mirroring the reference's tests/adapters/test_qwen15_moe_adapter.py. The kernels
themselves run in tests/test_gpu_hf_adapter.py."""
from __future__ import annotations

import pytest
import torch
from torch import nn


class FakeConfig:
    model_type = "qwen2_moe"
    architectures = ("Qwen2MoeForCausalLM",)
    num_experts_per_tok = 2


class SwiGLU(nn.Module):
    def __init__(self, H, I):
        super().__init__()
        self.gate_proj = nn.Linear(H, I, bias=False)
        self.up_proj = nn.Linear(H, I, bias=False)
        self.down_proj = nn.Linear(I, H, bias=False)


class FakeQwenMoeBlock(nn.Module):
    def __init__(self, H=256, E=4, I=128):
        super().__init__()
        self.gate = nn.Linear(H, E, bias=False)
        self.experts = nn.ModuleList([SwiGLU(H, I) for _ in range(E)])
        self.top_k = 2
        self.norm_topk_prob = True


class FakeQwenModel(nn.Module):
    def __init__(self, num_layers=2):
        super().__init__()
        self.config = FakeConfig()
        self.layers = nn.ModuleList([nn.Module() for _ in range(num_layers)])
        for layer in self.layers:
            layer.mlp = FakeQwenMoeBlock()


def _hf_tiny(norm_topk_prob=False):
    from transformers import Qwen2MoeConfig, Qwen2MoeForCausalLM

    cfg = Qwen2MoeConfig(vocab_size=64, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                         shared_expert_intermediate_size=256, num_hidden_layers=2, num_attention_heads=2,
                         num_key_value_heads=2, num_experts=8, num_experts_per_tok=2,
                         norm_topk_prob=norm_topk_prob, decoder_sparse_step=1, mlp_only_layers=[])
    return Qwen2MoeForCausalLM(cfg)


def test_discovers_module_list_layers(pkg):
    specs = pkg.hf_adapter.discover_moe_layers(FakeQwenModel())
    assert [s.name for s in specs] == ["layers.0.mlp", "layers.1.mlp"]
    s = specs[0]
    assert (s.num_experts, s.top_k, s.hidden_size, s.intermediate_size, s.layout) == (4, 2, 256, 128, "module_list")
    assert s.returns_router_logits and not s.has_shared_expert


def test_discovers_transformers_qwen2_moe_blocks(pkg):
    model = _hf_tiny()
    specs = pkg.hf_adapter.discover_moe_layers(model)
    assert len(specs) == 2
    s = specs[0]
    assert s.layout == "fused" and s.num_experts == 8 and s.top_k == 2 and s.intermediate_size == 128
    assert s.has_shared_expert and not s.returns_router_logits and s.norm_topk_prob is False
    assert pkg.hf_adapter.Qwen15MoEAdapter.supports(model)


def test_patch_and_restore(pkg):
    model = FakeQwenModel(num_layers=3)
    originals = [l.mlp for l in model.layers]
    ad = pkg.hf_adapter.Qwen15MoEAdapter(model)
    assert ad.patch_model() == 3
    assert all(type(l.mlp).__name__ == "B200MoEBlock" for l in model.layers)
    assert ad.patch_model() == 3  # idempotent
    assert ad.restore_model() == 3
    assert [l.mlp for l in model.layers] == originals


def test_unsupported_model_is_rejected(pkg):
    model = nn.Sequential(nn.Linear(4, 4))
    model.config = type("C", (), {"model_type": "dense"})()
    assert not pkg.hf_adapter.Qwen15MoEAdapter.supports(model)
    with pytest.raises(ValueError):
        pkg.hf_adapter.Qwen15MoEAdapter(model).patch_model()


def test_routing_mode_follows_norm_topk_prob(pkg):
    for norm, routing, want in ((True, "hf", 1), (False, "hf", 2), (False, "reference", 1)):
        model = _hf_tiny(norm_topk_prob=norm)
        ad = pkg.hf_adapter.Qwen15MoEAdapter(model, routing=routing)
        ad.patch_model()
        assert all(b.renormalize == want for b in ad.blocks)
    # the default is the reference's routing (softmax over the k selected), whatever the model says
    ad = pkg.hf_adapter.Qwen15MoEAdapter(_hf_tiny(norm_topk_prob=False))
    ad.patch_model()
    assert ad.routing == "reference" and all(b.renormalize == 1 for b in ad.blocks)


def test_cpu_forward_fails_loudly(pkg):
    model = FakeQwenModel(num_layers=1)
    pkg.hf_adapter.Qwen15MoEAdapter(model).patch_model()
    with pytest.raises(RuntimeError, match="CUDA"):
        model.layers[0].mlp(torch.randn(2, 256))


def test_dequantize_fp8_channel_and_block(pkg, orc):
    g = torch.Generator().manual_seed(3)
    w = torch.randn(256, 384, generator=g) * 0.02
    q, s = orc.quantize_channel(w)
    torch.testing.assert_close(pkg.hf_adapter.dequantize_fp8(q, s), orc.dequantize_channel(q, s))
    qb, sb = orc.quantize_blockwise(w)
    torch.testing.assert_close(pkg.hf_adapter.dequantize_fp8(qb, sb), orc.dequantize_blockwise(qb, sb))
    # re-quantising the dequantised weights reproduces every e4m3 code (amax = 448 * scale)
    q2, s2 = orc.quantize_channel(pkg.hf_adapter.dequantize_fp8(q, s))
    assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8))
    torch.testing.assert_close(s2, s, rtol=1e-6, atol=0)


def test_parallel_context_wiring(pkg):
    ha = pkg.hf_adapter
    with pytest.raises(ValueError):
        ha.ParallelContext(1, 0)
    with pytest.raises(ValueError):
        ha.ParallelContext(2, 2)
    model = _hf_tiny()
    ad = ha.Qwen15MoEAdapter(model, world_size=2, rank=1, ep_batch_size_threshold=32)
    ad.patch_model()
    ctx = ad.blocks[0].parallel
    assert ctx is not None and all(b.parallel is ctx for b in ad.blocks)
    assert (ctx.world, ctx.rank, ctx.threshold) == (2, 1, 32)
    assert ha.Qwen15MoEAdapter(_hf_tiny()).parallel is None

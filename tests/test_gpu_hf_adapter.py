"""HF adapter on the B200: a transformers Qwen2-MoE model (tiny, random init) patched
with B200MoEBlock against the unpatched model, the full-softmax routing mode, pre-quantised
e4m3 import, and the per-block CUDA graphs."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _tiny(norm_topk_prob, seed=0):
    from transformers import Qwen2MoeConfig, Qwen2MoeForCausalLM

    cfg = Qwen2MoeConfig(vocab_size=128, hidden_size=256, intermediate_size=512, moe_intermediate_size=256,
                         shared_expert_intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
                         num_key_value_heads=2, num_experts=8, num_experts_per_tok=2,
                         norm_topk_prob=norm_topk_prob, decoder_sparse_step=1, mlp_only_layers=[])
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    model = Qwen2MoeForCausalLM(cfg)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            elif "gate.weight" in name and p.ndim == 2 and p.shape[0] == 8:
                p.copy_(torch.randn(p.shape, generator=g) / p.shape[1] ** 0.5)  # router logits ~ N(0, 1)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    return model.to(DEV, torch.bfloat16).eval()


@pytest.mark.parametrize("norm_topk_prob", [False, True])
def test_router_modes_match_transformers(pkg, norm_topk_prob):
    from transformers.models.qwen2_moe import modeling_qwen2_moe as m

    model = _tiny(norm_topk_prob)
    blk = model.model.layers[0].mlp
    x = torch.randn(64, 256, device=DEV).bfloat16()
    _, w_hf, i_hf = blk.gate(x)
    res = pkg.ops.router_topk(x, blk.gate.weight.data, 2, renormalize=1 if norm_topk_prob else 2)
    # same expert sets (bf16 logits may tie: compare sets where the 2nd/3rd logits are apart)
    logits = (x.float() @ blk.gate.weight.float().t())
    top3 = logits.topk(3, dim=-1).values
    clear = (top3[:, 1] - top3[:, 2]) > 1e-2
    a = torch.sort(res.topk_indices, dim=-1).values[clear]
    b = torch.sort(i_hf, dim=-1).values[clear]
    assert torch.equal(a, b)
    # weights by expert id
    w_ours = torch.zeros(64, 8, device=DEV).scatter_(1, res.topk_indices, res.topk_weights)
    w_ref = torch.zeros(64, 8, device=DEV).scatter_(1, i_hf, w_hf.float())
    torch.testing.assert_close(w_ours[clear], w_ref[clear], rtol=2e-2, atol=2e-3)


def _clear_tokens(blk, x, gap=2e-2):
    """Tokens whose HF (bf16) router logits separate the k-th and (k+1)-th expert by > gap:
    on the others bf16 vs fp32 logits may legitimately pick another expert."""
    logits = torch.nn.functional.linear(x, blk.gate.weight).float()
    k = blk.gate.top_k
    top = logits.topk(k + 1, dim=-1).values
    return (top[:, k - 1] - top[:, k]) > gap


def _block_pair(pkg, model, layer, weight_dtype):
    spec = [s for s in pkg.hf_adapter.discover_moe_layers(model) if s.name == f"model.layers.{layer}.mlp"][0]
    ours = pkg.hf_adapter.B200MoEBlock(spec, weight_dtype=weight_dtype, routing="hf")  # vs transformers
    ours.prepare()
    return spec.module, ours


@pytest.mark.parametrize("norm_topk_prob", [False, True])
def test_bf16_block_matches_transformers_block(pkg, norm_topk_prob):
    model = _tiny(norm_topk_prob)
    hf, ours = _block_pair(pkg, model, 0, torch.bfloat16)
    x = torch.randn(1, 96, 256, generator=torch.Generator(device=DEV).manual_seed(1), device=DEV).bfloat16()
    with torch.no_grad():
        ref = hf(x)[0].float()
        out = ours(x)[0].float()
    m = _clear_tokens(hf, x[0])
    assert m.sum() > 80
    err = _rel(out[m], ref[m])
    assert err < 2e-2, f"rel Frobenius {err:.3e}"


def test_fp8_block_matches_transformers_block_on_the_same_weights(pkg):
    """FP8 block against the HF block whose expert weights are replaced by the dequantised
    e4m3 weights the kernels use."""
    model = _tiny(False, seed=3)
    hf, ours = _block_pair(pkg, model, 1, torch.float8_e4m3fn)
    I = 256
    with torch.no_grad():
        for e in range(8):
            g, u, d = ours.moe.experts.dequantized(e)
            hf.experts.gate_up_proj[e, :I].copy_(g)
            hf.experts.gate_up_proj[e, I:].copy_(u)
            hf.experts.down_proj[e].copy_(d)
        sg, su, sd = ours.moe.shared_expert.dequantized(0)
        hf.shared_expert.gate_proj.weight.copy_(sg)
        hf.shared_expert.up_proj.weight.copy_(su)
        hf.shared_expert.down_proj.weight.copy_(sd)
        x = torch.randn(1, 96, 256, generator=torch.Generator(device=DEV).manual_seed(2), device=DEV).bfloat16()
        ref = hf(x)[0].float()
        out = ours(x)[0].float()
    m = _clear_tokens(hf, x[0])
    err = _rel(out[m], ref[m])
    assert err < 2e-2, f"rel Frobenius {err:.3e}"


def test_patched_model_greedy_tokens_match_transformers(pkg):
    """Whole model (bf16 expert weights): next-token argmax agrees with the unpatched model
    on >= 90 % of positions (the reference validator's generated_token_parity idea), and
    restore_model brings back the original output bit for bit."""
    model = _tiny(False)
    ids = torch.randint(0, 128, (2, 24), generator=torch.Generator().manual_seed(1)).to(DEV)
    with torch.no_grad():
        ref = model(ids).logits.float()
    ad = pkg.hf_adapter.Qwen15MoEAdapter(model, weight_dtype=torch.bfloat16, routing="hf")
    assert ad.patch_model() == 2
    with torch.no_grad():
        out = model(ids).logits.float()
    agree = (out.argmax(-1) == ref.argmax(-1)).float().mean().item()
    assert agree >= 0.9, f"greedy agreement {agree:.2f}"
    ad.restore_model()
    with torch.no_grad():
        assert torch.equal(model(ids).logits.float(), ref)


@pytest.mark.parametrize("mode", ["channel", "block"])
def test_prequantized_import_reproduces_codes(pkg, orc, mode):
    H, I = 256, 256
    g = torch.Generator().manual_seed(7)
    mats = [torch.randn(I, H, generator=g) * 0.02, torch.randn(I, H, generator=g) * 0.02,
            torch.randn(H, I, generator=g) * 0.02]
    quant = orc.quantize_channel if mode == "channel" else orc.quantize_blockwise
    deq = orc.dequantize_channel if mode == "channel" else orc.dequantize_blockwise
    qs = [quant(w) for w in mats]
    sm = pkg._lib.SCALE_CHANNEL if mode == "channel" else pkg._lib.SCALE_BLOCK128
    store = pkg.ExpertWeightStore(1, H, I, weight_dtype=torch.float8_e4m3fn, scale_mode=sm, device=DEV)
    pkg.hf_adapter.import_fp8_expert(store, 0, *[t.to(DEV) for q in qs for t in q])
    for got, (q, s) in zip(store.dequantized(0), qs):
        torch.testing.assert_close(got.cpu(), deq(q, s), rtol=1e-6, atol=0)


def test_cuda_graph_blocks(pkg):
    model = _tiny(True, seed=5)
    ids = torch.randint(0, 128, (1, 16), generator=torch.Generator().manual_seed(4)).to(DEV)
    ad = pkg.hf_adapter.Qwen15MoEAdapter(model)
    ad.patch_model()
    with torch.no_grad():
        eager = model(ids).logits.float()
        assert ad.enable_cuda_graphs(warmup_steps=2) == 2
        g1 = model(ids).logits.float()
        g2 = model(ids).logits.float()
    st = ad.graph_statistics()
    assert st["captures"] == 2 and st["replays"] == 4 and st["fallbacks"] == 0
    assert torch.equal(g1, g2)
    assert _rel(g1, eager) < 1e-3


def _hybrid_worker(rank, world, port, q):
    import os

    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        global DEV
        DEV = f"cuda:{rank}"
        model = _tiny(True, seed=9)  # same weights on every rank
        ha = pkg.hf_adapter
        ctx = ha.ParallelContext(world, rank, ep_batch_size_threshold=16)
        specs = {s.name: s for s in ha.discover_moe_layers(model)}
        res = []
        for name in sorted(specs):  # same order on every rank: preparing is collective
            par = ha.B200MoEBlock(specs[name], parallel=ctx)
            ref = ha.B200MoEBlock(specs[name])
            par.prepare(dev)
            ref.prepare(dev)
            for T in (8, 96):  # EP below the threshold, DWDP above
                x = torch.randn(1, T, 256, generator=torch.Generator().manual_seed(50 + rank + T)).bfloat16().to(dev)
                with torch.no_grad():
                    y_par, y_ref = par(x), ref(x)
                torch.cuda.synchronize()
                st = par.ep_layer.read_status(T)[0] if T <= 16 else par.moe.read_status(T)[0]
                res.append((name, T, bool(torch.equal(y_par, y_ref)), st))
        dist.barrier()
        ctx.exchange.close()
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, repr(exc)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_hybrid_ep_dwdp_blocks_match_single_gpu():
    """world 2: each rank holds half of every block's experts; 8 tokens go the EP way, 96 the
    DWDP way; both must equal the single-GPU block bit for bit."""
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_hybrid_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in out:
        assert not isinstance(res, str), f"rank {rank}: {res}"
        for name, T, ok, st in res:
            assert st == 0, f"rank {rank} {name} T={T}: status {st}"
            assert ok, f"rank {rank} {name} T={T}: differs from the single-GPU block"

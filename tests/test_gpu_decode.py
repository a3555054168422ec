"""Decode-step parity on the B200: add_rmsnorm, rope_append_kv and paged_attention
against the CPU oracle (oracle/decode_oracle.py, pinned to transformers' Qwen2-MoE
modules), and a 2-layer Qwen-shaped decode step (eager and graph-replayed) against
the oracle composed with the MoE oracle under the step's own routing."""
from __future__ import annotations

import math

import pytest
import torch

from oracle import decode_oracle as dor

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_TOL = 5e-3  # rel Frobenius: bf16 output rounding of fp32 arithmetic
FP8_TOL = 2e-2


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("rows,H,with_delta", [(1, 2048, False), (37, 2048, True), (5, 7168, True)])
def test_add_rmsnorm(pkg, rows, H, with_delta):
    g = torch.Generator().manual_seed(rows + H)
    x = torch.randn(rows, H, generator=g).bfloat16()
    d = torch.randn(rows, H, generator=g).bfloat16() if with_delta else None
    w = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
    xr = x.to(DEV)
    out = pkg.ops.add_rmsnorm(xr, d.to(DEV) if d is not None else None, w.to(DEV), 1e-6)
    resid = (x.float() + d.float()).bfloat16() if with_delta else x
    assert torch.equal(xr.cpu(), resid)
    ref = dor.rms_norm(resid, w, 1e-6)
    assert _rel(out.cpu(), ref) < BF16_TOL


def _paged(B, NH, D, bs, max_blocks, g):
    nb = B * max_blocks + 3
    perm = torch.randperm(nb, generator=g)[: B * max_blocks].view(B, max_blocks).to(torch.int32)
    k = torch.randn(nb, bs, NH, D, generator=g).bfloat16()
    v = torch.randn(nb, bs, NH, D, generator=g).bfloat16()
    return perm, k, v


def _history(cache, table_row, n):
    """Positions [0, n) of one sequence, gathered from its pages: [n, NH, D]."""
    bs = cache.shape[1]
    rows = [cache[int(table_row[p // bs]), p % bs] for p in range(n)]
    return torch.stack(rows) if rows else cache.new_zeros(0, *cache.shape[2:])


def test_rope_append_kv(pkg):
    g = torch.Generator().manual_seed(11)
    B, NH, D, bs, mb = 4, 16, 128, 16, 8
    table, kc, vc = _paged(B, NH, D, bs, mb, g)
    qkv = torch.randn(B, 3 * NH * D, generator=g).bfloat16()
    bias = (0.1 * torch.randn(3 * NH * D, generator=g)).bfloat16()
    pos = torch.tensor([0, 5, 16, 127], dtype=torch.int32)
    kd, vd = kc.to(DEV), vc.to(DEV)
    st = torch.zeros(4, dtype=torch.int32, device=DEV)
    q = pkg.ops.rope_append_kv(qkv.to(DEV), bias.to(DEV), pos.to(DEV), table.to(DEV), kd, vd, 1e6, status=st)
    assert int(st[0]) == 0
    full = (qkv.float() + bias.float()).view(B, 3, NH, D)
    for b in range(B):
        p = int(pos[b])
        qr = dor.rope(full[b, 0][:, None, :], torch.tensor([p]), 1e6)[:, 0]
        kr = dor.rope(full[b, 1][:, None, :], torch.tensor([p]), 1e6)[:, 0]
        assert _rel(q[b].cpu(), qr) < BF16_TOL
        blk, off = int(table[b, p // bs]), p % bs
        assert _rel(kd[blk, off].cpu(), kr) < BF16_TOL
        assert torch.equal(vd[blk, off].cpu(), full[b, 2].bfloat16())
    # nothing else in the caches moved
    written = {(int(table[b, int(pos[b]) // bs]), int(pos[b]) % bs) for b in range(B)}
    mask = torch.ones(kc.shape[:2], dtype=torch.bool)
    for blk, off in written:
        mask[blk, off] = False
    assert torch.equal(kd.cpu()[mask], kc[mask]) and torch.equal(vd.cpu()[mask], vc[mask])


def test_rope_append_kv_bad_block_reports_status(pkg):
    NH, D, bs = 2, 128, 16
    table = torch.tensor([[0, -1]], dtype=torch.int32, device=DEV)
    kc = torch.zeros(2, bs, NH, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    st = torch.zeros(4, dtype=torch.int32, device=DEV)
    qkv = torch.randn(1, 3 * NH * D, device=DEV).bfloat16()
    pkg.ops.rope_append_kv(qkv, None, torch.tensor([20], dtype=torch.int32, device=DEV), table, kc, vc, 1e6,
                           status=st)
    torch.cuda.synchronize()
    assert int(st[0]) == pkg._lib.DWDP_ERR_DEVICE_BOUNDS
    assert int(kc.abs().sum()) == 0


@pytest.mark.parametrize("pos,table_row", [(40, [0, 1]), (-1, [0, 1]), (20, [0, 2]), (20, [0, 7])])
def test_rope_append_kv_out_of_range_reports_status(pkg, pos, table_row):
    """Positions past the block table (40 >= 2 * 16) or negative, and block ids past the cache
    (2 and 7 with 2 blocks): recorded in the status word, nothing written."""
    NH, D, bs = 2, 128, 16
    table = torch.tensor([table_row], dtype=torch.int32, device=DEV)
    kc = torch.zeros(2, bs, NH, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.zeros(1, NH, D, dtype=torch.bfloat16, device=DEV)
    st = torch.zeros(4, dtype=torch.int32, device=DEV)
    qkv = torch.randn(1, 3 * NH * D, device=DEV).bfloat16()
    pkg.ops.rope_append_kv(qkv, None, torch.tensor([pos], dtype=torch.int32, device=DEV), table, kc, vc, 1e6,
                           q_out=q, status=st)
    torch.cuda.synchronize()
    assert int(st[0]) == pkg._lib.DWDP_ERR_DEVICE_BOUNDS
    assert int(kc.abs().sum()) == 0 and int(vc.abs().sum()) == 0 and int(q.abs().sum()) == 0


@pytest.mark.parametrize("NH,bs", [(16, 16), (4, 16), (16, 6)])
@pytest.mark.parametrize("bad", [-1, 99])
def test_paged_attention_bad_block_skipped(pkg, NH, bs, bad):
    """A block id outside [0, num_blocks) on the bulk path (16 heads) and on the per-head
    fallback (4 heads; block size 6): recorded in the status word, and its positions are left
    out of the softmax, so the result equals attention over the other positions."""
    g = torch.Generator().manual_seed(23)
    D, mb = 128, 4
    table, kc, vc = _paged(1, NH, D, bs, mb, g)
    q = torch.randn(1, NH, D, generator=g).bfloat16()
    n = mb * bs
    bad_table = table.clone()
    bad_table[0, 1] = bad
    st = torch.zeros(4, dtype=torch.int32, device=DEV)
    out = pkg.ops.paged_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), bad_table.to(DEV),
                                  torch.tensor([n], dtype=torch.int32, device=DEV), n, status=st)
    torch.cuda.synchronize()
    assert int(st[0]) == pkg._lib.DWDP_ERR_DEVICE_BOUNDS
    keep = torch.ones(n, dtype=torch.bool)
    keep[bs:2 * bs] = False
    k = _history(kc, table[0], n)[keep]
    v = _history(vc, table[0], n)[keep]
    ref = dor.attention_decode(q[0], k, v, 1 / math.sqrt(D))
    assert _rel(out[0].cpu(), ref) < BF16_TOL


@pytest.mark.parametrize("NH,bs,splits", [(16, 16, 1), (16, 16, None), (16, 16, 37), (8, 16, None),
                                          (32, 16, None), (4, 16, None), (16, 6, None)])
def test_paged_attention_ragged(pkg, NH, bs, splits):
    """Bulk-copy path (8/16/32 heads, block_size % 4 == 0) and the per-head fallback."""
    g = torch.Generator().manual_seed(17)
    D = 128
    mb = -(-2048 // bs)
    lens = [1, 17, 300, 2048, 1000]
    B = len(lens)
    table, kc, vc = _paged(B, NH, D, bs, mb, g)
    q = torch.randn(B, NH, D, generator=g).bfloat16()
    out = pkg.ops.paged_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), table.to(DEV),
                                  torch.tensor(lens, dtype=torch.int32, device=DEV), 2048, splits=splits)
    for b, n in enumerate(lens):
        ref = dor.attention_decode(q[b], _history(kc, table[b], n), _history(vc, table[b], n), 1 / math.sqrt(D))
        assert _rel(out[b].cpu(), ref) < BF16_TOL, f"seq {b} (len {n})"


def test_paged_attention_matches_dense_softmax_at_scale(pkg):
    """B=64 sequences at the full 2048 context: against torch's fp32 attention on the GPU."""
    g = torch.Generator(device=DEV).manual_seed(3)
    B, NH, D, bs, mb = 64, 16, 128, 16, 128
    table = torch.randperm(B * mb, generator=g, device=DEV).view(B, mb).to(torch.int32)
    kc = torch.randn(B * mb, bs, NH, D, generator=g, device=DEV).bfloat16()
    vc = torch.randn(B * mb, bs, NH, D, generator=g, device=DEV).bfloat16()
    q = torch.randn(B, NH, D, generator=g, device=DEV).bfloat16()
    lens = torch.full((B,), 2048, dtype=torch.int32, device=DEV)
    out = pkg.ops.paged_attention(q, kc, vc, table, lens, 2048)
    k = kc[table.long()].view(B, mb * bs, NH, D).float()
    v = vc[table.long()].view(B, mb * bs, NH, D).float()
    s = torch.einsum("bhd,blhd->bhl", q.float(), k) / math.sqrt(D)
    ref = torch.einsum("bhl,blhd->bhd", torch.softmax(s, -1), v)
    assert _rel(out, ref) < BF16_TOL


def _small_cfg(pkg):
    return pkg.decode.QwenMoEConfig(vocab_size=512, num_layers=2, max_context=256)


def test_decode_step_matches_oracle(pkg, orc):
    cfg = _small_cfg(pkg)
    model = pkg.decode.QwenMoEDecodeModel(cfg, DEV, seed=99, max_batch=3)
    model.fill_context(seed=5)
    table = model.admit(3)
    tokens = torch.tensor([3, 400, 77])
    pos = torch.tensor([0, 100, 255], dtype=torch.int32)
    # pre-step cache copy: the oracle's history for positions < pos
    kv_before = model.cache.kv_cache.cpu()
    nxt = model.step(tokens, pos, table, graph=False)
    torch.cuda.synchronize()
    assert model.read_status(3)[0] == 0
    b = model.buffers(3)
    logits = b.logits.cpu()
    H, NH, D = cfg.hidden_size, cfg.num_heads, cfg.head_dim
    h = model.embed.cpu()[tokens].float()
    delta = None
    for l in range(cfg.num_layers):
        w = model.attn[l]
        if delta is not None:
            h = (h.bfloat16().float() + delta.bfloat16().float())
        h = h.bfloat16().float()
        outs = []
        for s in range(3):
            p = int(pos[s])
            kh = _history(kv_before[l, 0], table[s], p)
            vh = _history(kv_before[l, 1], table[s], p)
            o, knew, vnew = dor.decoder_attention_half(h[s], w.input_norm.cpu(), cfg.rms_norm_eps, kh, vh, p,
                                                       w.wqkv.cpu(), w.bqkv.cpu(), w.wo.cpu(), NH, cfg.rope_theta)
            blk, off = int(table[s, p // cfg.block_size]), p % cfg.block_size
            assert _rel(model.cache.k(l)[blk, off].cpu(), knew) < 1e-2
            outs.append(o)
        h = (h + torch.stack(outs).bfloat16().float()).bfloat16().float()
        xn = dor.rms_norm(h, w.post_norm.cpu(), cfg.rms_norm_eps).bfloat16()
        moe = model.moe[l]
        ws = b.moe_ws[l]
        idx, wts = ws.router.topk_indices.cpu(), ws.router.topk_weights.cpu()
        experts = [None] * moe.num_experts
        for e in sorted(set(idx.reshape(-1).tolist())):
            experts[e] = tuple(t.cpu() for t in moe.experts.dequantized(e))
        shared = tuple(t.cpu() for t in moe.shared_expert.dequantized(0))
        delta = orc.moe_forward(xn.float(), idx, wts, experts, shared=shared, shared_gate=ws.router.shared_gate.cpu())
    h = (h + delta.bfloat16().float()).bfloat16().float()
    ref = dor.rms_norm(h, model.final_norm.cpu(), cfg.rms_norm_eps).bfloat16().float() @ model.lm_head.cpu().float().t()
    assert _rel(logits, ref) < FP8_TOL
    # greedy token agrees wherever the oracle's top-2 logits are not within the tolerance
    top2 = ref.topk(2, dim=-1).values
    for s in range(3):
        if (top2[s, 0] - top2[s, 1]) > 0.05 * top2[s, 0].abs():
            assert int(nxt[s]) == int(ref[s].argmax())


def test_decode_step_graph_replay_equals_eager(pkg):
    cfg = _small_cfg(pkg)
    model = pkg.decode.QwenMoEDecodeModel(cfg, DEV, seed=7, max_batch=4)
    model.fill_context(seed=1)
    table = model.admit(4)
    tokens = torch.tensor([1, 2, 3, 4])
    pos = torch.tensor([10, 11, 200, 3], dtype=torch.int32)
    model.step(tokens, pos, table, graph=False)
    eager = model.buffers(4).logits.clone()
    model.step(tokens, pos, table, graph=True)  # capture + replay
    first = model.buffers(4).logits.clone()
    # cuBLAS may pick another algorithm under capture: equal to bf16 rounding, not bitwise
    assert _rel(first, eager) < 1e-3
    model.step(tokens, pos, table, graph=True)
    assert torch.equal(model.buffers(4).logits, first)
    # a new step position through the same graph: the cache slot it writes changes
    model.step(tokens, pos + 1, table, graph=True)
    torch.cuda.synchronize()
    assert not torch.equal(model.buffers(4).logits, eager)
    assert model.read_status(4)[0] == 0
    model.release(table)
    assert len(model.cache.free_blocks) == model.cache.num_blocks

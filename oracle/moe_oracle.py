"""CPU oracle for the DWDP MoE-layer hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or the timed CPU
baseline. The product path (the package's kernels) never calls it.

Each function restates the reference algorithm it cites (paths inside the DWDP
project). Integer work (dispatch) is plain Python loops or numpy and is meant to
be bit-exact; floating-point work uses torch on the CPU in fp32.

Pinning: ``tests/golden/`` holds vectors produced by running the reference
itself (``tests/golden/make_golden.py``) plus the hand-made golden cases of the
reference's own tests; ``tests/test_oracle_golden.py`` checks this module
against all of them.
"""
from __future__ import annotations

import numpy as np
import torch

FP8_E4M3_MAX = 448.0


# --------------------------------------------------------------------------- router
def router_logits(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                  score_scale: float = 1.0) -> torch.Tensor:
    """logits = x W^T (+ b), times score_scale, in fp32 (DWDP/router/linear.py:38-44)."""
    out = x.float() @ weight.float().T
    if bias is not None:
        out = out + bias.float()
    if score_scale != 1.0:
        out = out * score_scale
    return out


def topk_routing(logits: torch.Tensor, top_k: int, *, renormalize: bool = True,
                 eps: float = 1e-9) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Top-k over logits, softmax over the k selected, renormalise by
    sum.clamp_min(eps); k == 1 gives weight 1 (DWDP/router/kernels/fused.py:8-42,
    ops/topk.py:6-20, ops/softmax.py:6-21, ops/renorm.py:6-16).

    Slot order: descending logit, ties to the lower expert id (the reference's
    ``torch.topk(sorted=False)`` order is implementation-defined; the expert SET
    per token is what parity compares). Returns (probs, indices int64, weights)."""
    lg = logits.float()
    T, E = lg.shape
    order = np.argsort(-lg.numpy(), axis=1, kind="stable")[:, :top_k]
    idx = torch.from_numpy(order.astype(np.int64))
    vals = torch.gather(lg, 1, idx)
    probs = torch.softmax(vals, dim=-1)
    if top_k == 1:
        weights = torch.ones_like(probs)
    elif renormalize:
        weights = probs / probs.sum(dim=-1, keepdim=True).clamp_min(eps)
    else:
        weights = probs
    return probs, idx, weights


# --------------------------------------------------------------------------- dispatch
def counting_scatter_loop(flat_ids: list[int], num_experts: int, top_k: int) -> dict[str, list[int]]:
    """Pure-Python restatement of the reference host counting pass
    (DWDP/dispatcher/ops/scatter.py:6-34) and the scatters (:37-96). Small cases only."""
    counts = [0] * num_experts
    for e in flat_ids:
        counts[e] += 1
    offsets = [0] * (num_experts + 1)
    for e in range(num_experts):
        offsets[e + 1] = offsets[e] + counts[e]
    cursors = offsets[:-1].copy()
    dest = [0] * len(flat_ids)
    for i, e in enumerate(flat_ids):
        dest[i] = cursors[e]
        cursors[e] += 1
    n = len(flat_ids)
    perm = [0] * n
    ids = [0] * n
    tok = [0] * n
    for i, d in enumerate(dest):
        perm[d] = i
        ids[d] = flat_ids[i]
        tok[d] = i // top_k
    return {"counts": counts, "offsets": offsets, "perm": perm, "inv": dest, "ids": ids, "tok": tok}


def counting_scatter(flat_ids: np.ndarray, flat_weights: np.ndarray, num_experts: int,
                     top_k: int) -> dict[str, np.ndarray]:
    """Vectorised equivalent of :func:`counting_scatter_loop`: a stable sort by
    expert id gives the same destinations as the sequential cursor pass."""
    ids = np.asarray(flat_ids, dtype=np.int64)
    counts = np.bincount(ids, minlength=num_experts).astype(np.int64)
    offsets = np.zeros(num_experts + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    perm = np.argsort(ids, kind="stable").astype(np.int64)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(ids.size, dtype=np.int64)
    return {
        "counts": counts,
        "offsets": offsets,
        "perm": perm,
        "inv": inv,
        "ids": ids[perm],
        "tok": perm // top_k,
        "weights": np.asarray(flat_weights)[perm],
    }


def round_robin_schedule(counts: np.ndarray, offsets: np.ndarray, stream_count: int = 1) -> dict[str, np.ndarray]:
    """Active experts ascending (DWDP/scheduler/ops/round_robin.py:8-80)."""
    active = np.nonzero(np.asarray(counts) > 0)[0].astype(np.int64)
    order = np.arange(active.size, dtype=np.int64)
    return {
        "expert_queue": active,
        "expert_starts": np.asarray(offsets)[active],
        "expert_ends": np.asarray(offsets)[active + 1],
        "expert_counts": np.asarray(counts)[active],
        "execution_priority": order,
        "stream_assignments": order % stream_count,
    }


# --------------------------------------------------------------------------- weights
def quantize_blockwise(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (e4m3 [N, K], fp32 scales [ceil(N/128), ceil(K/128)]) with
    scale = max(amax of the 128x128 block, 1e-5) / 448 (DWDP/executor/fp8.py:118-146)."""
    N, K = w.shape
    nb, kb = -(-N // 128), -(-K // 128)
    work = torch.nn.functional.pad(w.float(), (0, kb * 128 - K, 0, nb * 128 - N))
    tiled = work.view(nb, 128, kb, 128)
    scales = tiled.abs().amax(dim=(1, 3)).clamp(min=1e-5) / FP8_E4M3_MAX
    q = (tiled / scales[:, None, :, None]).view(nb * 128, kb * 128)[:N, :K]
    return q.to(torch.float8_e4m3fn), scales.contiguous()


def quantize_channel(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel restatement of the same rule (no reference function):
    scale[n] = max(amax_k |w[n, k]|, 1e-5) / 448."""
    scales = w.float().abs().amax(dim=1).clamp(min=1e-5) / FP8_E4M3_MAX
    return (w.float() / scales[:, None]).to(torch.float8_e4m3fn), scales


def quantize_tensor(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """One scale per matrix: scale = max(amax |w|, 1e-5) / 448, q = e4m3(w / scale)
    (DWDP/executor/fp8.py:45-49, convert_qwen_weights_to_fp8_once with a scale_map).
    Returns (e4m3 [N, K], fp32 scalar tensor)."""
    scale = w.float().abs().max().clamp(min=1e-5) / FP8_E4M3_MAX
    return (w.float() / scale).to(torch.float8_e4m3fn), scale


def dequantize_tensor(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale


def dequantize_blockwise(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    N, K = q.shape
    s = scales.repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)[:, :K]
    return q.float() * s


def dequantize_channel(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    return q.float() * scales[:, None]


# --------------------------------------------------------------------------- experts + merge
def swiglu_expert(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                  *, round_intermediate: bool = False) -> torch.Tensor:
    """down(silu(gate x) * up x) in fp32 (the Qwen expert MLP the reference calls
    as ``module(x)``, DWDP/executor/pytorch.py:369-382). ``round_intermediate`` rounds the
    SwiGLU product to bf16 before the down projection, as a bf16 execution does."""
    x = x.float()
    h = torch.nn.functional.silu(x @ gate.float().T) * (x @ up.float().T)
    if round_intermediate:
        h = h.bfloat16().float()
    return h @ down.float().T


def swiglu_expert_fp8_act(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
                          down: torch.Tensor) -> torch.Tensor:
    """One expert as the reference's FP8 TMA executor computes it
    (DWDP/executor/triton_tma.py:185-207, kernels/fp8_tma.py:66-121), on dequantised
    weights: the activation rows are quantised to e4m3 with one scale per (row, 128
    channels) (DWDP/executor/fp8.py:86-115) and multiplied dequantised; gate and up
    outputs are rounded to bf16 (the executor's output dtype), the SwiGLU product is
    formed in bf16 (``gate * sigmoid(gate) * up``, each op rounded), re-quantised per
    (row, 128) the same way, and the down projection is rounded to bf16. A GEMM that
    promotes every 128-wide K block in fp32 (``acc += (Xq Wq^T)_kb * sx * sw``) equals
    this dequantised product up to fp32 summation order."""
    xq, xs = quantize_activations_blockwise(x)
    xd = dequantize_activations_blockwise(xq, xs)
    g = (xd @ gate.float().T).bfloat16()
    u = (xd @ up.float().T).bfloat16()
    h = g * torch.sigmoid(g) * u
    hq, hs = quantize_activations_blockwise(h.float())
    hd = dequantize_activations_blockwise(hq, hs)
    return (hd @ down.float().T).bfloat16().float()


def moe_forward(
    x: torch.Tensor,
    topk_idx: torch.Tensor,
    topk_weights: torch.Tensor,
    experts: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
    *,
    shared: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None,
    shared_gate: torch.Tensor | None = None,
    bf16_roundings: bool = False,
    act_quant: str = "none",
) -> torch.Tensor:
    """Routed experts in ascending expert order over the expert-major packing,
    weighted rows accumulated token-major (PyTorchExecutor + PyTorchMerger,
    DWDP/executor/pytorch.py:66-160, DWDP/merger/kernels/reference.py:6-27), then
    ``out += gate * shared(x)`` (DWDP/adapters/qwen15_moe.py:302-319). fp32 arithmetic;
    ``bf16_roundings`` applies the three roundings of a bf16 data path (SwiGLU intermediate,
    each weighted expert row, the output) so that only accumulation order differs.
    ``act_quant="block128"`` runs every expert (the shared one included) as the
    reference's FP8 executor does (:func:`swiglu_expert_fp8_act`), the weighted row
    rounded to bf16 as that executor's ``expert_out * weights`` is; ``experts`` may be
    any indexable whose item ``e`` is only looked up for experts the routing selects."""
    if act_quant not in ("none", "block128"):
        raise ValueError(f"unknown act_quant {act_quant!r}")
    fp8_act = act_quant == "block128"
    x = x.float()
    T, H = x.shape
    K = topk_idx.shape[-1]
    flat = topk_idx.reshape(-1).numpy()
    plan = counting_scatter(flat, topk_weights.reshape(-1).float().numpy(), len(experts), K)
    out = torch.zeros(T, H, dtype=torch.float32)
    for e in range(len(experts)):
        s, t = int(plan["offsets"][e]), int(plan["offsets"][e + 1])
        if s == t:
            continue
        tok = torch.from_numpy(plan["tok"][s:t])
        w = torch.from_numpy(np.ascontiguousarray(plan["weights"][s:t])).float()
        if fp8_act:
            y = (swiglu_expert_fp8_act(x[tok], *experts[e]).bfloat16() * w[:, None].bfloat16()).float()
        else:
            y = swiglu_expert(x[tok], *experts[e], round_intermediate=bf16_roundings) * w[:, None]
        if bf16_roundings:
            y = y.bfloat16().float()
        out.index_add_(0, tok, y)
    if shared is not None:
        ys = swiglu_expert_fp8_act(x, *shared) if fp8_act else \
            swiglu_expert(x, *shared, round_intermediate=bf16_roundings)
        if shared_gate is not None:
            ys = ys * shared_gate.float().reshape(-1, 1)
        if bf16_roundings:
            ys = ys.bfloat16().float()
        out = out + ys
    return out.bfloat16().float() if bf16_roundings else out


def rel_frobenius(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b||_F / ||b||_F in fp64."""
    a64, b64 = a.double(), b.double()
    den = b64.norm().item()
    return (a64 - b64).norm().item() / (den if den > 0 else 1.0)


def quantize_activations_blockwise(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (e4m3 [M, K], fp32 scales [M, ceil(K/128)]), one scale per
    (row, 128-column block) = max(amax, 1e-5) / 448 (DWDP/executor/fp8.py:86-115)."""
    M, K = x.shape
    kb = -(-K // 128)
    work = torch.nn.functional.pad(x.float(), (0, kb * 128 - K)).view(M, kb, 128)
    scales = work.abs().amax(dim=-1).clamp(min=1e-5) / FP8_E4M3_MAX
    q = (work / scales.unsqueeze(-1)).view(M, kb * 128)[:, :K]
    return q.to(torch.float8_e4m3fn), scales.contiguous()


def dequantize_activations_blockwise(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`quantize_activations_blockwise`: q * scale of its (row, 128) block."""
    M, K = q.shape
    return q.float() * scales.repeat_interleave(128, 1)[:, :K]

"""MoE layer forward on B200: router -> dispatch (+row gather) -> grouped tcgen05
expert GEMMs (routed + shared) -> deterministic merge.

This is the fused equivalent of one ``DWDPMoEBlock`` eager forward
(DWDP/adapters/qwen15_moe.py:350-431: router, dispatcher, scheduler, executor,
merger, then ``_add_shared_expert`` at :302-319) and of ``DWDPRuntime.forward``
(DWDP/runtime/runtime.py:189-275) without the Python per-expert loop: a fixed
sequence of this library's launches per layer and no host synchronisation, so
the whole call can be captured in a CUDA graph.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .weights import ExpertWeightStore


@dataclass
class LayerWorkspace:
    """Per-token-count scratch owned by the layer (never returned to callers)."""

    num_tokens: int
    router: ops.RouterResult
    dispatch: ops.DispatchResult
    dispatch_scratch: torch.Tensor
    weighted: torch.Tensor
    shared_out: torch.Tensor | None
    shared_parts: int
    moe_ws: torch.Tensor
    status: torch.Tensor
    shared_ws: torch.Tensor | None = None        # the shared expert's own launches (side stream)
    side: torch.cuda.Stream | None = None
    ticket: torch.Tensor | None = None           # one-launch router + dispatch (decode sizes)
    gate_logit: torch.Tensor | None = None


class MoELayer:
    """One MoE layer: ``E`` routed SwiGLU experts (top-k over the router logits,
    softmax over the k selected, optional renormalisation) plus an optional
    sigmoid-gated shared expert. Activations are bf16; weights are fp8
    (per-channel, per-tensor or 128x128 block scales) or bf16, held in an
    ExpertWeightStore. ``activation_quant`` ("hilo" or "block128", see
    ExpertWeightStore) chooses how the e4m3 GEMMs carry the activations."""

    def __init__(
        self,
        router_weight: torch.Tensor,
        experts: ExpertWeightStore,
        top_k: int,
        *,
        shared_expert: ExpertWeightStore | None = None,
        shared_gate_weight: torch.Tensor | None = None,
        router_bias: torch.Tensor | None = None,
        renormalize: bool = True,
        eps: float = 1e-9,
        score_scale: float = 1.0,
        activation_quant: str | None = None,
    ) -> None:
        E, H = router_weight.shape
        if experts.num_experts != E or experts.hidden_size != H:
            raise ValueError("router weight and expert store disagree on E or H")
        if shared_expert is not None and (shared_expert.num_experts != 1 or shared_expert.hidden_size != H):
            raise ValueError("shared expert store must hold exactly one expert of the same hidden size")
        if top_k <= 0 or top_k > E:
            raise ValueError("top_k must be in [1, num_experts]")
        self.router_weight = router_weight.contiguous()
        self.router_bias = router_bias
        self.experts = experts
        self.shared_expert = shared_expert
        self.shared_gate_weight = shared_gate_weight
        self.top_k = top_k
        self.renormalize = renormalize
        self.eps = eps
        self.score_scale = score_scale
        # e4m3 activation scheme of both groups' GEMMs (the store's own setting unless given)
        self.activation_quant = activation_quant or getattr(experts, "activation_quant", None) or \
            getattr(getattr(experts, "local", None), "activation_quant", "hilo")
        self.num_experts = E
        self.hidden_size = H
        self._ws: dict[int, LayerWorkspace] = {}
        # The shared expert does not depend on routing, so it CAN run on a side stream from
        # the start of the forward. Measured slower on B200 at T = 1..4096 (the persistent
        # GEMMs each size their grid to every SM, so concurrent launches queue behind each
        # other, and the cross-stream join breaks the programmatic-launch chain): off by default.
        self.overlap_shared = False
        # the smallest decode sizes (ops.use_fused_routing): router and dispatch in one launch
        self.fused_routing = True
        self.refresh_handles()

    def refresh_handles(self) -> None:
        """Rebuild the C handles (call after swapping pointer-array tensors)."""
        aq = self.activation_quant
        self._routed_group = self.experts.group(aq)
        self._shared_group = self.shared_expert.group(aq) if self.shared_expert is not None else None

    # ------------------------------------------------------------------ workspace
    def workspace(self, num_tokens: int) -> LayerWorkspace:
        ws = self._ws.get(num_tokens)
        if ws is not None:
            return ws
        T, K, E, H = num_tokens, self.top_k, self.num_experts, self.hidden_size
        N = T * K
        dev = self.router_weight.device
        has_shared = self.shared_expert is not None
        router = ops.RouterResult(
            router_logits=torch.empty(T, E, dtype=torch.float32, device=dev),
            routing_probabilities=torch.empty(T, K, dtype=torch.float32, device=dev),
            topk_indices=torch.empty(T, K, dtype=torch.int64, device=dev),
            topk_weights=torch.empty(T, K, dtype=torch.float32, device=dev),
            shared_gate=torch.empty(T, dtype=torch.float32, device=dev)
            if (has_shared and self.shared_gate_weight is not None) else None,
        )
        disp = ops.DispatchResult(
            expert_counts=torch.empty(E, dtype=torch.int64, device=dev),
            expert_offsets=torch.empty(E + 1, dtype=torch.int64, device=dev),
            token_permutation=torch.empty(N, dtype=torch.int64, device=dev),
            inverse_permutation=torch.empty(N, dtype=torch.int64, device=dev),
            packed_expert_ids=torch.empty(N, dtype=torch.int64, device=dev),
            packed_token_indices=torch.empty(N, dtype=torch.int64, device=dev),
            packed_routing_weights=torch.empty(N, dtype=torch.float32, device=dev),
            packed_hidden=None,  # the expert kernels read hidden through packed_token_indices
        )
        Is = self.shared_expert.intermediate_size if has_shared else 0
        parts = ops.moe_shared_parts(T, Is) if has_shared else 0
        ws = LayerWorkspace(
            num_tokens=T,
            router=router,
            dispatch=disp,
            dispatch_scratch=torch.empty(ops.dispatch_scratch_bytes(T, K, E), dtype=torch.uint8, device=dev),
            weighted=torch.empty(N, H, dtype=torch.bfloat16, device=dev),
            shared_out=torch.empty(parts, T, H, dtype=torch.bfloat16, device=dev) if has_shared else None,
            shared_parts=parts,
            moe_ws=torch.empty(
                ops.moe_workspace_bytes(T, K, E, self.experts.intermediate_size, Is),
                dtype=torch.uint8, device=dev,
            ),
            status=torch.zeros(4, dtype=torch.int32, device=dev),
            shared_ws=torch.empty(ops.moe_shared_workspace_bytes(T, H, Is), dtype=torch.uint8, device=dev)
            if has_shared else None,
            side=torch.cuda.Stream(device=dev) if has_shared else None,
            ticket=torch.zeros(1, dtype=torch.int32, device=dev),
            gate_logit=torch.empty(max(T, 1), dtype=torch.float32, device=dev),
        )
        self._ws[num_tokens] = ws
        return ws

    # ------------------------------------------------------------------ forward
    def forward(self, hidden_states: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        """hidden [..., H] bf16 -> MoE output [..., H] bf16 (a fresh tensor unless
        ``out`` is given; it never aliases the layer workspace)."""
        if hidden_states.dtype != torch.bfloat16:
            raise ValueError("MoELayer expects bf16 hidden states")
        H = self.hidden_size
        if hidden_states.shape[-1] != H:
            raise ValueError(f"hidden size {hidden_states.shape[-1]} != {H}")
        token_shape = hidden_states.shape[:-1]
        x = hidden_states.reshape(-1, H).contiguous()
        T = x.shape[0]
        if out is None:
            out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
        if T == 0:
            return out.reshape(*token_shape, H)
        self.run(x, self.workspace(T), out)
        return out.reshape(*token_shape, H)

    __call__ = forward

    def run(self, x: torch.Tensor, ws: LayerWorkspace, out: torch.Tensor) -> None:
        """All launches on the current stream, the shared expert's on the workspace's side
        stream joined before the merge (graph-capturable)."""
        K = self.top_k
        T = x.shape[0]
        overlap = self._overlap(ws)
        if overlap:
            self._start_shared(x, ws)
        gate_w = self.shared_gate_weight if self.shared_expert is not None else None
        if self.fused_routing and ops.use_fused_routing(T, K, self.num_experts, x, self.router_weight):
            # decode sizes: router and dispatch in one launch
            ops.route_dispatch_small(x, self.router_weight, K, ws.router, ws.dispatch, ws.ticket, ws.gate_logit,
                                     bias=self.router_bias, shared_gate_weight=gate_w, score_scale=self.score_scale,
                                     renormalize=self.renormalize, eps=self.eps, status=ws.status)
        else:
            ops.router_topk(
                x, self.router_weight, K, bias=self.router_bias, shared_gate_weight=gate_w,
                score_scale=self.score_scale, renormalize=self.renormalize, eps=self.eps, out=ws.router,
            )
            # the expert kernels read routed rows through packed_token_indices: no gathered copy
            ops.dispatch(
                ws.router.topk_indices, ws.router.topk_weights, self.num_experts,
                scratch=ws.dispatch_scratch, out=ws.dispatch, status=ws.status,
            )
        self._routed(x, ws, with_shared=not overlap)
        if overlap:
            torch.cuda.current_stream().wait_stream(ws.side)
            ops.merge(ws.weighted, ws.dispatch.inverse_permutation, T, K, shared_out=ws.shared_out,
                      shared_parts=ws.shared_parts, out=out, shared_gate=ws.router.shared_gate)
        else:
            ops.merge(ws.weighted, ws.dispatch.inverse_permutation, T, K, shared_out=ws.shared_out,
                      shared_parts=ws.shared_parts, out=out)

    def run_experts(self, x: torch.Tensor, ws: LayerWorkspace) -> None:
        """Every expert GEMM of :meth:`run` on a dispatched workspace (weighted rows and
        shared partials; the shared ones ungated when they run on the side stream)."""
        overlap = self._overlap(ws)
        if overlap:
            self._start_shared(x, ws)
        self._routed(x, ws, with_shared=not overlap)
        if overlap:
            torch.cuda.current_stream().wait_stream(ws.side)

    def _overlap(self, ws: LayerWorkspace) -> bool:
        return self.overlap_shared and ws.side is not None

    def _start_shared(self, x: torch.Tensor, ws: LayerWorkspace) -> None:
        ws.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(ws.side):
            ops.moe_shared_expert(self._shared_group, x, ws.shared_out, ws.shared_ws, ws.status)

    def _routed(self, x: torch.Tensor, ws: LayerWorkspace, *, with_shared: bool) -> None:
        ops.moe_experts(
            self._routed_group, self._shared_group if with_shared else None, None, x, self.top_k,
            ws.dispatch.expert_counts, ws.dispatch.expert_offsets, ws.dispatch.packed_routing_weights,
            ws.router.shared_gate if with_shared else None, ws.weighted,
            ws.shared_out if with_shared else None, ws.moe_ws, ws.status,
            packed_token_indices=ws.dispatch.packed_token_indices,
        )

    def kernel_launches(self, num_tokens: int) -> int:
        """Kernels one forward launches: router (1 for bf16 weights, else logits +
        top-k), dispatch (scatter, plus a histogram above 256 assignments), expert
        plan (+ activation planes), [row gather,] gate/up GEMM, [intermediate
        planes,] down GEMM, merge."""
        router = 1 if self.router_weight.dtype == torch.bfloat16 and self.num_experts <= 256 else 2
        dispatch = 1 if num_tokens * self.top_k <= 256 else 2
        if (self.fused_routing and self.router_weight.dtype == torch.bfloat16 and self.num_experts <= 256
                and 0 < num_tokens <= ops.FUSED_ROUTING_MAX_TOKENS and num_tokens * self.top_k <= 256):
            router, dispatch = 1, 0
        # e4m3 hi/lo: plan(+planes), gate/up, planes, down; e4m3 block128: the gate/up epilogue
        # writes the intermediate's e4m3 rows, so no launch between the GEMMs; bf16: row gather
        fp8 = self.experts.weight_dtype == torch.float8_e4m3fn
        experts = 3 if (fp8 and self.activation_quant == "block128") else 4
        if self.shared_expert is not None and self.overlap_shared:
            experts += experts  # the shared expert's own launches
        return router + dispatch + experts + 1

    def read_status(self, num_tokens: int) -> tuple[int, ...]:
        """Device status word {code, where, detail, count} of the last forward."""
        return tuple(self.workspace(num_tokens).status.cpu().tolist())


def algorithmic_bytes(layer: MoELayer, counts: torch.Tensor, num_tokens: int) -> int:
    """Minimum bytes one forward must move: weights + scales of the active experts
    and the shared expert, router weight, activations in/out, routing indices."""
    active = int((counts > 0).sum().item())
    b = active * layer.experts.nbytes_per_expert()
    if layer.shared_expert is not None:
        b += layer.shared_expert.nbytes_per_expert() + layer.hidden_size * 2
    b += layer.router_weight.numel() * layer.router_weight.element_size()
    b += num_tokens * layer.hidden_size * 2 * 2
    b += num_tokens * layer.top_k * (8 + 4)
    return b


def algorithmic_flops(layer: MoELayer, num_tokens: int) -> int:
    """2*T*K*3*H*I (routed) + 2*T*3*H*Is (shared) + 2*T*H*E (router)."""
    H, I, K, E = layer.hidden_size, layer.experts.intermediate_size, layer.top_k, layer.num_experts
    f = 2 * num_tokens * K * 3 * H * I + 2 * num_tokens * H * E
    if layer.shared_expert is not None:
        f += 2 * num_tokens * 3 * H * layer.shared_expert.intermediate_size
    return f

"""Hugging Face adapter: swap the sparse-MoE blocks of a Qwen1.5/Qwen2-MoE model for
blocks backed by this library's kernels.

Mirrors the reference adapter (``DWDP/adapters/qwen15_moe.py:434-580``: ``supports``,
``patch_model``, ``restore_model``, ``enable_cuda_graphs``, ``graph_statistics``; layer
discovery ``DWDP/adapters/extractor.py``; module swapping ``DWDP/adapters/patcher.py``)
with two model layouts:

* the layout the reference targets: ``block.gate`` an ``nn.Linear`` [E, H] and
  ``block.experts`` an ``nn.ModuleList`` of SwiGLU experts with ``gate_proj`` /
  ``up_proj`` / ``down_proj`` linears; the block returns ``(hidden, router_logits)``;
* transformers 5.x ``Qwen2MoeSparseMoeBlock``: ``block.gate`` a top-k router holding
  ``weight`` [E, H] and ``block.experts`` one module with fused ``gate_up_proj``
  [E, 2I, H] and ``down_proj`` [E, H, I] parameters; the block returns the hidden
  states alone.

Weights are imported once per block (lazily, on the block's first forward or on
``adapter.prepare()``): bf16/fp32 experts are quantised to e4m3 with per-output-channel
(or 128x128 block) scales, or kept bf16; experts that are already e4m3 with their scale
tensors (``weight_scale`` / ``weight_scale_inv`` attributes, per output channel or per
128x128 block) are imported from those (``import_fp8_expert``). Routing defaults to the
reference's (``routing="reference"``, DWDP/router/kernels/fused.py:25-35): the softmax
over the k selected, whatever the replaced module's ``norm_topk_prob`` says, so a block
swapped in for the reference's ``DWDPMoEBlock`` gives the reference's outputs.
``routing="hf"`` follows the replaced transformers module instead: ``norm_topk_prob``
true gives the softmax over the k selected; false gives the selected experts'
probabilities under the softmax over all experts (what transformers computes).

With ``world_size > 1`` (one process per GPU, ``torch.distributed`` initialised) every block
holds only its rank's shard of the experts and runs the reference's hybrid
(``DWDP/adapters/qwen15_moe.py:325-345``): batches above ``ep_batch_size_threshold`` tokens per
rank prefetch the remote experts over NVLink (DWDP), smaller ones exchange token rows with the
expert owners (EP); see ``ParallelContext``.

There is no CPU execution: a patched block raises ``RuntimeError`` off CUDA.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
from torch import nn

from . import _lib
from .layer import MoELayer
from .weights import ExpertWeightStore


# --------------------------------------------------------------------------- discovery
@dataclass
class MoELayerSpec:
    """One discovered sparse-MoE block (DWDP/adapters/extractor.py:9-23)."""

    name: str
    module: nn.Module
    parent: nn.Module
    child_name: str
    gate_weight: torch.Tensor  # [E, H]
    gate_bias: torch.Tensor | None
    layout: str  # "module_list" | "fused"
    hidden_size: int
    num_experts: int
    intermediate_size: int
    top_k: int
    norm_topk_prob: bool
    has_shared_expert: bool
    returns_router_logits: bool


def _parent(root: nn.Module, qualified: str) -> tuple[nn.Module, str]:
    parts = qualified.split(".")
    mod = root
    for p in parts[:-1]:
        mod = getattr(mod, p)
    return mod, parts[-1]


def _config_top_k(config: Any) -> int | None:
    for attr in ("num_experts_per_tok", "num_experts_per_token", "moe_top_k", "top_k"):
        v = getattr(config, attr, None)
        if v is not None:
            return int(v)
    return None


def _swiglu_expert(e: nn.Module) -> bool:
    return all(isinstance(getattr(e, n, None), nn.Linear) for n in ("gate_proj", "up_proj", "down_proj"))


def discover_moe_layers(model: nn.Module) -> tuple[MoELayerSpec, ...]:
    """Sparse-MoE blocks of a Qwen-style HF model whose experts this library can run."""
    config = getattr(model, "config", None)
    specs = []
    for name, module in model.named_modules():
        if not name or not any(k in name for k in ("mlp", "moe", "block", "layer")):
            continue
        gate, experts = getattr(module, "gate", None), getattr(module, "experts", None)
        if gate is None or experts is None:
            continue
        gw = getattr(gate, "weight", None)
        if not isinstance(gw, torch.Tensor) or gw.ndim != 2:
            continue
        top_k = getattr(module, "top_k", None) or getattr(gate, "top_k", None) or _config_top_k(config)
        if top_k is None:
            continue
        norm = getattr(module, "norm_topk_prob", getattr(gate, "norm_topk_prob", None))
        if norm is None:
            norm = bool(getattr(config, "norm_topk_prob", True))
        if isinstance(experts, (nn.ModuleList, list, tuple)):
            if len(experts) == 0 or not all(_swiglu_expert(e) for e in experts):
                continue
            layout, I = "module_list", experts[0].gate_proj.out_features
        elif isinstance(getattr(experts, "gate_up_proj", None), torch.Tensor) and \
                isinstance(getattr(experts, "down_proj", None), torch.Tensor):
            layout, I = "fused", experts.gate_up_proj.shape[1] // 2
        else:
            continue
        parent, child = _parent(model, name)
        specs.append(MoELayerSpec(
            name=name, module=module, parent=parent, child_name=child, gate_weight=gw,
            gate_bias=getattr(gate, "bias", None), layout=layout, hidden_size=int(gw.shape[1]),
            num_experts=int(gw.shape[0]), intermediate_size=int(I), top_k=int(top_k), norm_topk_prob=bool(norm),
            has_shared_expert=getattr(module, "shared_expert", None) is not None,
            returns_router_logits=isinstance(gate, nn.Linear)))
    return tuple(specs)


# --------------------------------------------------------------------------- weight import
def _fp8_scale(linear_or_param: Any) -> torch.Tensor | None:
    for attr in ("weight_scale", "weight_scale_inv", "scale"):
        s = getattr(linear_or_param, attr, None)
        if isinstance(s, torch.Tensor):
            return s
    return None


def _fused_scale(experts: nn.Module, name: str) -> torch.Tensor | None:
    """Scale tensor of a fused e4m3 expert parameter: a sibling ``<name>_scale`` /
    ``<name>_scale_inv`` / ``<name>_weight_scale`` tensor, or one attached to the parameter."""
    for suffix in ("_scale", "_scale_inv", "_weight_scale"):
        s = getattr(experts, name + suffix, None)
        if isinstance(s, torch.Tensor):
            return s
    return _fp8_scale(getattr(experts, name))


def dequantize_fp8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3 [R, C] with a per-row [R] / [R, 1] scale or a [ceil(R/128), ceil(C/128)] block
    scale -> fp32."""
    R, C = q.shape
    qf = q.float()
    s = scale.float().to(q.device)
    if s.numel() == R:
        return qf * s.reshape(R, 1)
    if s.ndim == 2 and s.shape == (-(-R // 128), -(-C // 128)):
        return qf * s.repeat_interleave(128, 0)[:R].repeat_interleave(128, 1)[:, :C]
    raise ValueError(f"unsupported fp8 scale shape {tuple(scale.shape)} for weight {tuple(q.shape)}")


def import_fp8_expert(store: ExpertWeightStore, e: int, gate_q: torch.Tensor, gate_s: torch.Tensor,
                      up_q: torch.Tensor, up_s: torch.Tensor, down_q: torch.Tensor, down_s: torch.Tensor) -> None:
    """Load one pre-quantised expert. A checkpoint quantised with scale = amax / 448 (per
    output channel, or per 128x128 block into a BLOCK128 store) is reproduced code for code:
    the dequantised row (block) has amax = 448 * scale, so re-quantising returns every e4m3
    code unchanged and the scale to within fp32 rounding."""
    store.load_expert(e, dequantize_fp8(gate_q, gate_s), dequantize_fp8(up_q, up_s), dequantize_fp8(down_q, down_s))


def _expert_mats(spec: MoELayerSpec, e: int):
    """(gate, up, down) of expert e as ([I,H], [I,H], [H,I]) tensors, or the e4m3 codes
    with their scales when the checkpoint is pre-quantised."""
    ex = spec.module.experts
    if spec.layout == "module_list":
        m = ex[e]
        mats = (m.gate_proj, m.up_proj, m.down_proj)
        ws = [lin.weight for lin in mats]
        if ws[0].dtype == torch.float8_e4m3fn:
            return "fp8", [(w, _fp8_scale(lin)) for w, lin in zip(ws, mats)]
        return "dense", ws
    I = spec.intermediate_size
    gu, dn = ex.gate_up_proj[e], ex.down_proj[e]
    if gu.dtype == torch.float8_e4m3fn:
        sgu, sdn = _fused_scale(ex, "gate_up_proj"), _fused_scale(ex, "down_proj")
        if sgu is None or sdn is None:
            raise ValueError(f"{spec.name}: e4m3 experts without scale tensors")
        sgu, sdn = sgu[e], sdn[e]
        half = sgu.shape[0] // 2
        return "fp8", [(gu[:I], sgu[:half]), (gu[I:], sgu[half:]), (dn, sdn)]
    return "dense", [gu[:I], gu[I:], dn]


def _load_expert(load, spec: MoELayerSpec, e: int, device) -> None:
    """load(e, gate, up, down) with expert e's weights (dequantised first when pre-quantised)."""
    kind, mats = _expert_mats(spec, e)
    if kind == "fp8":
        (gq, gs), (uq, us), (dq, ds) = mats
        if gs is None or us is None or ds is None:
            raise ValueError(f"{spec.name}: e4m3 expert {e} without scale tensors")
        load(e, dequantize_fp8(gq.to(device), gs), dequantize_fp8(uq.to(device), us),
             dequantize_fp8(dq.to(device), ds))
    else:
        load(e, *(t.detach().to(device) for t in mats))


def _store_from(spec: MoELayerSpec, weight_dtype: torch.dtype, scale_mode: int, device) -> ExpertWeightStore:
    store = ExpertWeightStore(spec.num_experts, spec.hidden_size, spec.intermediate_size, weight_dtype=weight_dtype,
                              scale_mode=scale_mode if weight_dtype == torch.float8_e4m3fn else _lib.SCALE_NONE,
                              device=device)
    for e in range(spec.num_experts):
        _load_expert(store.load_expert, spec, e, device)
    return store


def _sharded_store_from(spec: MoELayerSpec, weight_dtype: torch.dtype, scale_mode: int, device, rank: int,
                        world: int, group=None):
    """This rank's shard (owner(e) = e // ceil(E / G)) of the block's experts, connected to the
    other ranks' shards (collective over ``group``)."""
    from .dwdp import ShardedExpertStore

    store = ShardedExpertStore(spec.num_experts, spec.hidden_size, spec.intermediate_size, rank=rank,
                               world_size=world, weight_dtype=weight_dtype,
                               scale_mode=scale_mode if weight_dtype == torch.float8_e4m3fn else _lib.SCALE_NONE,
                               device=device, num_buffers=1)
    for e in store.owned:
        _load_expert(store.load_expert, spec, e, device)
    store.connect(group)
    return store


def _shared_store(module: nn.Module, weight_dtype, scale_mode, device) -> ExpertWeightStore | None:
    sh = getattr(module, "shared_expert", None)
    if sh is None:
        return None
    if not _swiglu_expert(sh):
        raise ValueError("shared expert must be a SwiGLU MLP with gate_proj/up_proj/down_proj")
    I, H = sh.gate_proj.out_features, sh.gate_proj.in_features
    store = ExpertWeightStore(1, H, I, weight_dtype=weight_dtype,
                              scale_mode=scale_mode if weight_dtype == torch.float8_e4m3fn else _lib.SCALE_NONE,
                              device=device)
    store.load_expert(0, *(lin.weight.detach().to(device) for lin in (sh.gate_proj, sh.up_proj, sh.down_proj)))
    return store


# --------------------------------------------------------------------------- graph runner
@dataclass
class GraphStats:
    captures: int = 0
    replays: int = 0
    fallbacks: int = 0
    shapes: list = field(default_factory=list)


class BlockGraphRunner:
    """Shape-keyed CUDA graph of one block's forward (DWDP/runtime/cuda_graph.py:63-201):
    warm-up on a side stream, capture at the first call of each token count, replay after;
    inputs are copied into a static buffer, the output buffer is the graph's own (the
    caller gets a copy). Shapes that fail to capture run eagerly (counted as fallbacks)."""

    def __init__(self, fn, warmup_steps: int = 3):
        self.fn = fn
        self.warmup_steps = max(1, warmup_steps)
        self.stats = GraphStats()
        self._graphs: dict[tuple, tuple] = {}
        self._failed: set[tuple] = set()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        key = (tuple(x.shape), x.dtype, x.device)
        if key in self._failed:
            self.stats.fallbacks += 1
            return self.fn(x)
        entry = self._graphs.get(key)
        if entry is None:
            try:
                entry = self._capture(x)
            except RuntimeError:
                self._failed.add(key)
                self.stats.fallbacks += 1
                return self.fn(x)
            self._graphs[key] = entry
            self.stats.captures += 1
            self.stats.shapes.append(tuple(x.shape))
        graph, xin, yout = entry
        xin.copy_(x)
        graph.replay()
        self.stats.replays += 1
        return yout.clone()

    def _capture(self, x: torch.Tensor):
        xin = x.clone()
        s = torch.cuda.Stream(device=x.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(self.warmup_steps):
                self.fn(xin)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            yout = self.fn(xin)
        return graph, xin, yout


# --------------------------------------------------------------------------- multi-GPU
class ParallelContext:
    """Expert parallelism across ``world`` ranks for every patched block of a model (the
    reference's hybrid, DWDP/adapters/qwen15_moe.py:325-345): each rank holds its shard of
    every block's experts; batches of more than ``ep_batch_size_threshold`` tokens per rank
    prefetch the remote experts over NVLink (DWDP), smaller ones send their token rows to the
    owners and back (EP, one exchange buffer shared by all blocks). Every rank must run the
    same blocks in the same order with the same token count."""

    def __init__(self, world_size: int, rank: int, *, ep_batch_size_threshold: int = 64, group=None) -> None:
        if world_size < 2 or not 0 <= rank < world_size:
            raise ValueError("ParallelContext needs world_size >= 2 and 0 <= rank < world_size")
        self.world, self.rank, self.group = world_size, rank, group
        self.threshold = ep_batch_size_threshold
        self.exchange = None

    def exchange_for(self, hidden_size: int, top_k: int, device):
        from .ep import EPExchange

        if self.exchange is None:
            self.exchange = EPExchange(self.world, self.rank, hidden_size, self.threshold, top_k, device)
            self.exchange.connect(self.group)
        elif (self.exchange.H, self.exchange.top_k) != (hidden_size, top_k):
            raise ValueError("every patched block must share the hidden size and top_k")
        return self.exchange


# --------------------------------------------------------------------------- the block
class B200MoEBlock(nn.Module):
    """Drop-in for a Qwen-style sparse-MoE block (DWDP/adapters/qwen15_moe.py:43-323):
    router -> dispatch -> grouped e4m3 GEMMs -> merge (+ sigmoid-gated shared expert) in this
    library's kernels. The router weight is shared with the replaced module when it already
    is a contiguous bf16 CUDA tensor."""

    def __init__(self, spec: MoELayerSpec, *, weight_dtype: torch.dtype = torch.float8_e4m3fn,
                 scale_mode: int = _lib.SCALE_CHANNEL, routing: str = "reference",
                 parallel: ParallelContext | None = None) -> None:
        super().__init__()
        if routing not in ("hf", "reference"):
            raise ValueError("routing must be 'hf' or 'reference'")
        self.spec = spec
        self.layer_name = spec.name
        self.hidden_size = spec.hidden_size
        self.num_experts = spec.num_experts
        self.top_k = spec.top_k
        self.returns_router_logits = spec.returns_router_logits
        self.weight_dtype = weight_dtype
        self.scale_mode = scale_mode
        self.renormalize = 1 if (spec.norm_topk_prob or routing == "reference") else 2
        self.moe: MoELayer | None = None
        self.parallel = parallel
        self.ep_layer = None  # the EP path of this block (multi-GPU, small batches)
        self._graph_runner: BlockGraphRunner | None = None

    def prepare(self, device: torch.device | str | None = None) -> MoELayer:
        """Import the weights (once) onto ``device`` (default: where the router weight is)."""
        if self.moe is not None:
            return self.moe
        dev = torch.device(device) if device is not None else self.spec.gate_weight.device
        if dev.type != "cuda":
            raise RuntimeError("B200MoEBlock runs on CUDA only (no CPU fallback); move the model to a GPU")
        spec, mod = self.spec, self.spec.module
        router_w = spec.gate_weight.detach().to(dev, torch.bfloat16).contiguous()
        bias = spec.gate_bias.detach().to(dev).float() if spec.gate_bias is not None else None
        gate_lin = getattr(mod, "shared_expert_gate", None)
        gate_w = gate_lin.weight.detach().to(dev, torch.bfloat16).reshape(-1) if gate_lin is not None else None
        shared = _shared_store(mod, self.weight_dtype, self.scale_mode, dev)
        par = self.parallel
        if par is None:
            store = _store_from(spec, self.weight_dtype, self.scale_mode, dev)
        else:
            store = _sharded_store_from(spec, self.weight_dtype, self.scale_mode, dev, par.rank, par.world, par.group)
            from .ep import ExpertParallelMoE

            self.ep_layer = ExpertParallelMoE(router_w, store.local, spec.top_k,
                                              par.exchange_for(spec.hidden_size, spec.top_k, dev),
                                              shared_expert=shared, shared_gate_weight=gate_w, router_bias=bias,
                                              renormalize=self.renormalize)
        self.moe = MoELayer(router_w, store, spec.top_k, shared_expert=shared, shared_gate_weight=gate_w,
                            router_bias=bias, renormalize=self.renormalize)
        return self.moe

    def _use_ep(self, num_tokens: int) -> bool:
        return self.ep_layer is not None and num_tokens <= self.parallel.threshold

    @property
    def router_weight(self) -> torch.Tensor:
        return self.prepare().router_weight

    def _run(self, x: torch.Tensor) -> torch.Tensor:
        if self._use_ep(x.shape[0]):
            return self.ep_layer(x)
        if self.parallel is not None:  # DWDP: the remote experts into staging, then the GEMMs
            self.moe.experts.prefetch(0)
            self.moe.experts.wait(0)
        return self.moe(x)

    def forward(self, hidden_states: torch.Tensor, *args, **kwargs):
        del args, kwargs
        if not hidden_states.is_cuda:
            raise RuntimeError("B200MoEBlock runs on CUDA only (no CPU fallback)")
        moe = self.prepare(hidden_states.device)
        shape, dtype = hidden_states.shape, hidden_states.dtype
        x = hidden_states.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        T = x.shape[0]
        # graphs replay the single-GPU and EP paths; the DWDP prefetch runs eagerly
        graph = self._graph_runner is not None and (self.parallel is None or self._use_ep(T))
        y = self._graph_runner(x) if graph else self._run(x)
        out = y.to(dtype).reshape(shape)
        if self.returns_router_logits:
            router = self.ep_layer.workspace(T)["router"] if self._use_ep(T) else moe.workspace(T).router
            logits = router.router_logits.to(dtype, copy=True)
            return out, logits.reshape(*shape[:-1], self.num_experts)
        return out

    def enable_cuda_graphs(self, warmup_steps: int = 3) -> bool:
        if not torch.cuda.is_available():
            return False
        self._graph_runner = BlockGraphRunner(self._run, warmup_steps=warmup_steps)
        return True


# --------------------------------------------------------------------------- the adapter
class Qwen15MoEAdapter:
    """Patch / restore the MoE blocks of a Qwen1.5/Qwen2-MoE HF model
    (DWDP/adapters/qwen15_moe.py:434-580)."""

    def __init__(self, model: nn.Module, *, weight_dtype: torch.dtype = torch.float8_e4m3fn,
                 scale_mode: int = _lib.SCALE_CHANNEL, routing: str = "reference", world_size: int = 1, rank: int = 0,
                 ep_batch_size_threshold: int = 64, group=None) -> None:
        self.model = model
        self.parallel = (ParallelContext(world_size, rank, ep_batch_size_threshold=ep_batch_size_threshold,
                                         group=group) if world_size > 1 else None)
        self.weight_dtype = weight_dtype
        self.scale_mode = scale_mode
        self.routing = routing
        self.moe_layer_specs: tuple[MoELayerSpec, ...] = ()
        self._records: list[tuple[MoELayerSpec, nn.Module, B200MoEBlock]] = []

    @classmethod
    def supports(cls, model: Any) -> bool:
        cfg = getattr(model, "config", None)
        names = " ".join([str(getattr(cfg, "model_type", "")), type(model).__name__,
                          *(str(a) for a in (getattr(cfg, "architectures", ()) or ()))]).lower()
        return "qwen" in names and bool(discover_moe_layers(model))

    def patch_model(self) -> int:
        if self._records:
            return len(self._records)
        specs = discover_moe_layers(self.model)
        if not specs:
            raise ValueError("no supported Qwen MoE layers were discovered")
        self.moe_layer_specs = specs
        for spec in specs:
            block = B200MoEBlock(spec, weight_dtype=self.weight_dtype, scale_mode=self.scale_mode,
                                 routing=self.routing, parallel=self.parallel)
            setattr(spec.parent, spec.child_name, block)
            self._records.append((spec, spec.module, block))
        return len(specs)

    @property
    def blocks(self) -> list[B200MoEBlock]:
        return [b for _, _, b in self._records]

    def prepare(self) -> int:
        """Import every patched block's weights now instead of at its first forward."""
        for b in self.blocks:
            b.prepare()
        return len(self._records)

    def restore_model(self) -> int:
        n = 0
        for spec, original, _ in reversed(self._records):
            setattr(spec.parent, spec.child_name, original)
            n += 1
        self._records.clear()
        return n

    def enable_cuda_graphs(self, warmup_steps: int = 3) -> int:
        if not self._records:
            raise RuntimeError("patch_model() must run before enabling CUDA graphs")
        return sum(int(b.enable_cuda_graphs(warmup_steps)) for b in self.blocks)

    def graph_statistics(self) -> dict[str, int]:
        tot = {"captures": 0, "replays": 0, "fallbacks": 0}
        for b in self.blocks:
            r = b._graph_runner
            if r is not None:
                for k in tot:
                    tot[k] += getattr(r.stats, k)
        return tot

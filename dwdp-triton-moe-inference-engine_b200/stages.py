"""Stage operators with the reference's interfaces, backed by the B200 kernels.

Each class keeps the constructor and ``forward`` signature of the reference
stage it stands in for, and returns the dataclasses of :mod:`plans`:

============================== ==========================================================
``B200LinearTopKRouter``       DWDP/router/linear.py:16-95 ``LinearTopKRouter``
``B200ExpertMajorDispatcher``  DWDP/dispatcher/expert_major.py:20-90
``B200RoundRobinScheduler``    DWDP/scheduler/policies/round_robin.py:17-89
``StaticCommunicationPlanner`` DWDP/comms_planner/static.py:27-110 (all experts local)
``B200Executor``               DWDP/executor/base.py:25-36 ``BaseExecutor.forward``
``B200Merger``                 DWDP/merger/pytorch.py:16-104 ``PyTorchMerger``
``B200Runtime``                DWDP/runtime/runtime.py:76-275 ``build_reference`` / ``forward``
============================== ==========================================================

Registries mirror ``register_*`` / ``build_*`` of the reference's per-stage
``registry.py`` modules; every B200 class is registered under a ``b200_*`` name.
None of these stages computes on the CPU: CUDA tensors are required.
"""
from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass

import torch
from torch import nn

from . import _lib, ops
from .plans import (EXECUTION_STATISTICS_FIELDS, SCHEDULER_STATISTICS_FIELDS, CommunicationPlan,
                    DependencyMetadata, DispatchMetadata, DispatchPlan, ExecutionMetadata, ExecutionPlan,
                    ExecutorOutput, ExpertAssignments, LazyStatistics, MergeMetadata, MergerOutput,
                    MergeStatistics, OutputMetadata, RouterOutput, RoutingMetadata, SynchronizationMetadata,
                    TimingMetadata, WorkspaceMetadata)
from .weights import ExpertWeightStore

# ----------------------------------------------------------------------------- registries
_REGISTRIES: dict[str, dict[str, type]] = {k: {} for k in
                                           ("router", "dispatcher", "scheduler", "planner", "executor", "merger")}


def _register(kind: str, name: str, cls: type) -> None:
    reg = _REGISTRIES[kind]
    if name in reg:
        raise ValueError(f"{kind.capitalize()} '{name}' is already registered")
    reg[name] = cls


def _lookup(kind: str, name: str) -> type:
    try:
        return _REGISTRIES[kind][name]
    except KeyError as exc:
        raise KeyError(f"Unknown {kind} type '{name}'") from exc


def register_router(name: str, cls: type) -> None:
    _register("router", name, cls)


def register_dispatcher(name: str, cls: type) -> None:
    _register("dispatcher", name, cls)


def register_scheduler(name: str, cls: type) -> None:
    _register("scheduler", name, cls)


def register_communication_planner(name: str, cls: type) -> None:
    _register("planner", name, cls)


def register_executor(name: str, cls: type) -> None:
    _register("executor", name, cls)


def register_merger(name: str, cls: type) -> None:
    _register("merger", name, cls)


# ----------------------------------------------------------------------------- configs
@dataclass(frozen=True, slots=True)
class RouterConfig:
    """Subset of DWDP/router/config.py:17-50 that the B200 router honours."""

    hidden_size: int
    num_experts: int
    top_k: int
    bias: bool = False
    router_type: str = "b200_linear_topk"
    renormalize: bool = True
    metadata_level: str = "counts"
    score_scale: float = 1.0
    eps: float = 1e-9
    shared_gate: bool = False
    weight_dtype: torch.dtype = torch.bfloat16

    def __post_init__(self) -> None:
        if self.hidden_size <= 0:
            raise ValueError("hidden_size must be > 0")
        if self.num_experts <= 0:
            raise ValueError("num_experts must be > 0")
        if self.top_k <= 0:
            raise ValueError("top_k must be > 0")
        if self.top_k > self.num_experts:
            raise ValueError("top_k must be <= num_experts")
        if self.score_scale <= 0.0:
            raise ValueError("score_scale must be > 0")
        if self.eps <= 0.0:
            raise ValueError("eps must be > 0")


@dataclass(frozen=True, slots=True)
class DispatcherConfig:
    """DWDP/dispatcher/config.py:8-39 with the B200 algorithm name."""

    num_experts: int
    dispatcher_type: str = "b200_expert_major"
    algorithm: str = "b200_counting_scatter"
    stable_order: bool = True
    reuse_router_metadata: bool = True
    validate_inputs: bool = False  # the reference's checks read values back to the host
    index_dtype: torch.dtype = torch.int64

    def __post_init__(self) -> None:
        if self.num_experts <= 0:
            raise ValueError("num_experts must be > 0")
        if self.index_dtype is not torch.int64:
            raise ValueError("The B200 dispatcher requires torch.int64 indices")
        if not self.stable_order:
            raise ValueError(f"{self.algorithm} requires stable_order=True")


@dataclass(frozen=True, slots=True)
class SchedulerConfig:
    scheduling_policy: str = "b200_round_robin"
    deterministic: bool = True
    stream_count: int = 1

    def __post_init__(self) -> None:
        if self.stream_count <= 0:
            raise ValueError("stream_count must be > 0")


@dataclass(frozen=True, slots=True)
class CommunicationPlannerConfig:
    """DWDP/comms_planner/config.py:15-60 (the fields the planners read)."""

    planner_policy: str = "static"
    world_size: int = 1
    local_rank: int = 0
    local_gpu_id: int | None = None  # None: the local rank
    deterministic: bool = True
    default_link_bandwidth_gbps: float = 0.0
    default_link_latency_us: float = 0.0

    def __post_init__(self) -> None:
        if self.world_size <= 0:
            raise ValueError("world_size must be > 0")
        if not 0 <= self.local_rank < self.world_size:
            raise ValueError("local_rank must satisfy 0 <= local_rank < world_size")


@dataclass(frozen=True, slots=True)
class ExecutorConfig:
    """DWDP/executor/config.py:8-38 plus the weight format of the B200 store."""

    backend: str = "b200"
    weight_dtype: torch.dtype = torch.float8_e4m3fn
    scale_mode: int = _lib.SCALE_CHANNEL
    deterministic: bool = True
    materialize_packed_outputs: bool = False
    # drive the grouped GEMMs from a TensorList built from the plans (tensor_list.py)
    # instead of the store's per-expert pointer arrays; same kernels, same results
    use_tensor_list: bool = False


@dataclass(frozen=True, slots=True)
class MergerConfig:
    backend: str = "b200"
    apply_routing_weights: bool = False
    deterministic: bool = True
    out_dtype: torch.dtype = torch.bfloat16


# ----------------------------------------------------------------------------- router
class B200LinearTopKRouter(nn.Module):
    """logits = x W^T (+b) (*score_scale) in fp32, top-k over logits, softmax over
    the k, renormalisation; counts/offsets metadata come from the dispatcher."""

    def __init__(self, config: RouterConfig) -> None:
        super().__init__()
        self.config = config
        wdt = getattr(config, "weight_dtype", torch.bfloat16)
        self.weight = nn.Parameter(torch.empty(config.num_experts, config.hidden_size, dtype=wdt))
        self.bias = nn.Parameter(torch.zeros(config.num_experts)) if config.bias else None
        self.shared_gate_weight = (nn.Parameter(torch.zeros(config.hidden_size, dtype=wdt))
                                   if getattr(config, "shared_gate", False) else None)
        nn.init.xavier_uniform_(self.weight)

    @property
    def num_experts(self) -> int:
        return self.config.num_experts

    @property
    def top_k(self) -> int:
        return self.config.top_k

    def _route(self, flat: torch.Tensor) -> ops.RouterResult:
        return ops.router_topk(flat, self.weight.detach(), self.config.top_k,
                               bias=None if self.bias is None else self.bias.detach(),
                               shared_gate_weight=None if self.shared_gate_weight is None
                               else self.shared_gate_weight.detach(),
                               score_scale=self.config.score_scale, renormalize=self.config.renormalize,
                               eps=self.config.eps)

    def compute_router_logits(self, flat_hidden_states: torch.Tensor) -> torch.Tensor:
        return self._route(flat_hidden_states).router_logits

    def forward(self, hidden_states: torch.Tensor, metadata_level: str | None = None) -> RouterOutput:
        H = self.config.hidden_size
        if hidden_states.shape[-1] != H:
            raise ValueError(f"hidden_states last dimension must be {H}")
        token_shape = tuple(hidden_states.shape[:-1])
        flat = hidden_states.reshape(-1, H)
        r = self._route(flat)
        level = str(getattr(metadata_level or self.config.metadata_level, "value",
                            metadata_level or self.config.metadata_level))
        md = None
        if level != "none":
            md = RoutingMetadata(num_tokens=flat.shape[0], num_experts=self.config.num_experts,
                                 top_k=self.config.top_k)
        E, K = self.config.num_experts, self.config.top_k
        return RouterOutput(
            router_logits=r.router_logits.reshape(*token_shape, E),
            routing_probabilities=r.routing_probabilities.reshape(*token_shape, K),
            topk_indices=r.topk_indices.reshape(*token_shape, K),
            topk_weights=r.topk_weights.reshape(*token_shape, K),
            metadata=md,
            shared_gate=r.shared_gate,
        )


# ----------------------------------------------------------------------------- dispatcher
class B200ExpertMajorDispatcher(nn.Module):
    """Bit-exact stable counting-sort dispatch (DWDP/dispatcher/kernels/reference.py:163-257)."""

    def __init__(self, config: DispatcherConfig) -> None:
        super().__init__()
        self.config = config

    @property
    def num_experts(self) -> int:
        return self.config.num_experts

    def forward(self, router_output: RouterOutput, workspace=None,
                hidden_states: torch.Tensor | None = None) -> DispatchPlan:
        idx, w = router_output.topk_indices, router_output.topk_weights
        if idx.shape != w.shape:
            raise ValueError("topk_indices and topk_weights must have identical shapes")
        if self.config.validate_inputs and idx.numel() > 0:
            lo, hi = int(idx.min().item()), int(idx.max().item())
            if lo < 0 or hi >= self.config.num_experts:
                raise ValueError(f"topk_indices contain out-of-range expert ids: [{lo}, {hi}]")
        K = idx.shape[-1]
        token_shape = tuple(idx.shape[:-1])
        r = ops.dispatch(idx, w, self.config.num_experts, hidden=hidden_states)
        N = idx.numel()
        md = DispatchMetadata(
            num_tokens=N // K, num_assignments=N, num_experts=self.config.num_experts, top_k=K,
            token_shape=token_shape, expert_counts=r.expert_counts, expert_offsets=r.expert_offsets,
            token_permutation=r.token_permutation, inverse_permutation=r.inverse_permutation,
            destination_positions=r.inverse_permutation, stable_order=True, algorithm=self.config.algorithm)
        if router_output.metadata is not None:
            router_output.metadata.tokens_per_expert = r.expert_counts
            router_output.metadata.expert_offsets = r.expert_offsets
        return DispatchPlan(
            assignments=ExpertAssignments(expert_ids=r.packed_expert_ids,
                                          packed_token_indices=r.packed_token_indices,
                                          packed_routing_weights=r.packed_routing_weights),
            metadata=md, packed_hidden=r.packed_hidden)


# ----------------------------------------------------------------------------- scheduler / planner
class B200RoundRobinScheduler(nn.Module):
    def __init__(self, config: SchedulerConfig) -> None:
        super().__init__()
        self.config = config

    def forward(self, dispatch_plan: DispatchPlan, workspace=None) -> ExecutionPlan:
        md = dispatch_plan.metadata
        r = ops.schedule(md.expert_counts, md.expert_offsets, self.config.stream_count)
        dev = r.expert_queue.device
        counts, policy = md.expert_counts, self.config.scheduling_policy

        def stats() -> dict:  # DWDP/scheduler/policies/round_robin.py _build_statistics, read on demand
            c = counts.cpu()
            active = c[c > 0]
            n_act = int(active.numel())
            return dict(num_experts=int(c.numel()), num_active_experts=n_act,
                        num_empty_experts=int(c.numel()) - n_act, num_execution_batches=n_act,
                        num_assignments=md.num_assignments,
                        max_tokens_per_expert=int(active.max()) if n_act else 0,
                        min_tokens_per_active_expert=int(active.min()) if n_act else 0, scheduling_policy=policy)

        empty = torch.empty(0, dtype=torch.int64, device=dev)
        return ExecutionPlan(execution_order=r.execution_priority, expert_queue=r.expert_queue,
                             expert_starts=r.expert_starts, expert_ends=r.expert_ends,
                             expert_counts=r.expert_counts, execution_priority=r.execution_priority,
                             stream_assignments=r.stream_assignments, batches=(),
                             synchronization=SynchronizationMetadata(
                                 barrier_after_batch=torch.empty(0, dtype=torch.bool, device=dev)),
                             dependencies=DependencyMetadata(dependency_src=empty, dependency_dst=empty),
                             statistics=LazyStatistics(stats, SCHEDULER_STATISTICS_FIELDS),
                             scheduling_policy=policy, deterministic=self.config.deterministic,
                             num_active=r.num_active)


def _planner_gpu(config) -> int:
    g = getattr(config, "local_gpu_id", None)
    return getattr(config, "local_rank", 0) if g is None else g


def _empty_plan_parts(dev, config, *, world_size: int, fabric: str, domains: tuple, locality: tuple,
                      connectivity=None):
    from . import comms_metadata as cmd

    e64 = torch.empty(0, device=dev, dtype=torch.int64)
    topo = cmd.TopologyMetadata(
        local_gpu_id=_planner_gpu(config), world_size=world_size, local_rank=getattr(config, "local_rank", 0),
        gpu_ids=torch.arange(world_size, device=dev, dtype=torch.int64),
        numa_domains=torch.zeros(world_size, device=dev, dtype=torch.int64), nvlink_connectivity=connectivity,
        nvswitch_domains=None, pcie_hierarchy=None, communication_domains=domains, locality_groups=locality,
        fabric=fabric, default_link_bandwidth_gbps=getattr(config, "default_link_bandwidth_gbps", 0.0),
        default_link_latency_us=getattr(config, "default_link_latency_us", 0.0))
    return e64, topo


class StaticCommunicationPlanner(nn.Module):
    """Every expert local (DWDP/comms_planner/static.py:37-110): the full plan schema with no
    descriptors, an empty graph and a zero cost model."""

    def __init__(self, config: CommunicationPlannerConfig | None = None) -> None:
        super().__init__()
        self.config = config or CommunicationPlannerConfig()

    def forward(self, execution_plan: ExecutionPlan, workspace=None,
                num_experts: int | None = None) -> CommunicationPlan:
        from . import comms_metadata as cmd
        from . import cost_model as cm

        dev = execution_plan.expert_queue.device
        E = num_experts if num_experts is not None else execution_plan.expert_queue.numel()
        G = getattr(self.config, "world_size", 1)
        gpu = _planner_gpu(self.config)
        e64, topo = _empty_plan_parts(
            dev, self.config, world_size=G, fabric="single_gpu" if G == 1 else "unspecified",
            domains=(cmd.CommunicationDomain(0, "local", (gpu,), getattr(self.config, "default_link_bandwidth_gbps", 0.0),
                                             getattr(self.config, "default_link_latency_us", 0.0)),),
            locality=((gpu,),))
        f32 = torch.empty(0, device=dev, dtype=torch.float32)
        local = torch.arange(E, device=dev, dtype=torch.int64)
        policy = self.config.planner_policy
        return CommunicationPlan(
            local_expert_ids=local, remote_expert_ids=e64,
            graph=cmd.CommunicationGraph((), (), e64, e64, e64), topology=topo,
            synchronization=cmd.SynchronizationMetadata(e64, e64, e64, e64),
            dependencies=cmd.DependencyMetadata(e64, e64, e64), prefetch=cmd.PrefetchPlan(e64, e64, f32),
            overlap=cmd.OverlapPlan(e64, e64, f32),
            cost_model=cm.CommunicationCostModel((), 0, 0.0, 0.0, 0.0),
            statistics=cmd.CommunicationStatistics(E, 0, 0, 0, 0, 0, 0, 0.0, policy),
            planner_policy=policy, deterministic=getattr(self.config, "deterministic", True))


SLICE_BYTES = 2 * 1024 * 1024  # the reference's NVLink slice (expert_parallel.py:60, buffers.cu kSliceSize)


class DWDPCommunicationPlanner(nn.Module):
    """DWDP weight-streaming plan (DWDP/comms_planner/expert_parallel.py:182-359): experts
    sharded over the ranks by owner(e) = e // ceil(E / G) (:120-122); the local rank's experts
    stay local, every other one is planned as 2 MiB slice descriptors whose start slice is
    rotated by the local rank (slice (rank + i) % n first, so ranks reading one peer enter its
    memory at different offsets), priority E - position among the remote experts, one group
    per source GPU, and the prefetch list with those priorities. ``op_type`` is
    ``p2p_weight_copy`` where the owner is peer-reachable, else ``staged_weight_copy``.

    Where the reference fills its cost model with constants, the estimates here come from a
    measured ``LinkProfile`` (``cost_model.measure_link``) and the prefetch window the caller
    expects (the previous layer's compute time); without one they carry the config's default
    link figures like the reference's. ``bytes_per_expert`` is an int or a callable e -> bytes
    (the reference reads it from its GlobalExpertTable; 0 = unknown gives one empty
    descriptor per expert, as there). ``peer_access(src, dst)`` defaults to the driver's
    peer-access query. ``slice_bytes = 0`` plans one descriptor per expert. Issue order is
    the engine's TransferScheduler's (``CommunicationEngine.execute_plan``)."""

    def __init__(self, config: CommunicationPlannerConfig | None = None, *, link=None,
                 bytes_per_expert=0, prefetch_window_us: float = 0.0, peer_access=None,
                 slice_bytes: int = SLICE_BYTES) -> None:
        super().__init__()
        self.config = config or CommunicationPlannerConfig(planner_policy="dwdp")
        self.link = link
        self.bytes_per_expert = bytes_per_expert
        self.prefetch_window_us = prefetch_window_us
        self.peer_access = peer_access
        self.slice_bytes = int(slice_bytes)

    def _expert_bytes(self, e: int) -> int:
        b = self.bytes_per_expert
        return int(b(e) if callable(b) else b)

    def _can_access(self, src: int, dst: int) -> bool:
        if src == dst:
            return True
        if self.peer_access is not None:
            return bool(self.peer_access(src, dst))
        try:
            from .communication import PeerTopology

            return PeerTopology().can_access(src, dst)
        except Exception:  # no driver here: treat the peer as unreachable (staged copy)
            return False

    def forward(self, execution_plan: ExecutionPlan, workspace=None,
                num_experts: int | None = None) -> CommunicationPlan:
        from . import comms_metadata as cmd
        from . import cost_model as cm
        from .dwdp import owner_of

        cfg = self.config
        dev = execution_plan.expert_queue.device
        E = num_experts if num_experts is not None else execution_plan.expert_queue.numel()
        G, r = cfg.world_size, cfg.local_rank
        gpu = _planner_gpu(cfg)
        owners = [owner_of(e, E, G) for e in range(E)]
        local = [e for e in range(E) if owners[e] == r]
        remote = [e for e in range(E) if owners[e] != r]
        bw = getattr(cfg, "default_link_bandwidth_gbps", 0.0)
        lat = getattr(cfg, "default_link_latency_us", 0.0)
        descs, transfers, pf_ids, pf_prio = [], [], [], []
        for position, e in enumerate(remote):
            owner, size = owners[e], self._expert_bytes(e)
            step = self.slice_bytes if self.slice_bytes > 0 else max(size, 1)
            n = max(1, -(-size // step))
            op = "p2p_weight_copy" if self._can_access(owner, gpu) else "staged_weight_copy"
            prio = E - position
            for i in range(n):
                off = ((r + i) % n) * step
                nb = min(step, size - off) if size else 0
                d = len(descs)
                descs.append(cmd.CommunicationDescriptor(d, op, owner, gpu, e, e, off, off + nb, nb, prio, 1))
                transfers.append(cmd.TransferDescriptor(d, d, owner, gpu, e, e, nb, prio))
            pf_ids.append(e)
            pf_prio.append(prio)
        if self.link is not None:
            model = cm.build_descriptor_cost_model(descs, self.link, prefetch_window_us=self.prefetch_window_us)
        else:  # the reference's constant-filled model (expert_parallel.py:248-260, 298-304)
            model = cm.CommunicationCostModel(
                estimates=tuple(cm.CommunicationCostEstimate(d.descriptor_id, d.count, lat, bw, d.priority,
                                                             0.0, 0.0, 0.0, 0.0) for d in descs),
                total_estimated_bytes=sum(d.count for d in descs), total_estimated_latency_us=0.0,
                critical_path_us=0.0, estimated_bandwidth_gbps=bw)
        i64 = lambda v: torch.tensor(v, device=dev, dtype=torch.int64)  # noqa: E731
        groups = tuple(cmd.CommunicationGroup(gi, i64([d.descriptor_id for d in descs if d.source_gpu == src]),
                                              src, gpu, 0, 0)
                       for gi, src in enumerate(sorted({d.source_gpu for d in descs})))
        peers = tuple(g for g in range(G) if self._can_access(g, gpu))
        conn = torch.zeros(G, G, device=dev, dtype=torch.int64)
        for s_ in range(G):
            for d_ in range(G):
                if self._can_access(s_, d_):
                    conn[d_, s_] = 1
        e64, topo = _empty_plan_parts(
            dev, cfg, world_size=G, fabric="nvlink" if G > 1 else "single_gpu",
            domains=(cmd.CommunicationDomain(0, "nvlink" if len(peers) > 1 else "local", peers or (gpu,), bw, lat),),
            locality=(peers or (gpu,),), connectivity=conn)
        node_ids = i64([d.descriptor_id for d in descs])
        f32 = torch.empty(0, device=dev, dtype=torch.float32)
        policy = cfg.planner_policy
        return CommunicationPlan(
            local_expert_ids=i64(local), remote_expert_ids=i64(remote),
            graph=cmd.CommunicationGraph((), (), node_ids, e64, e64),
            communication_descriptors=tuple(descs), transfer_descriptors=tuple(transfers),
            communication_groups=groups, topology=topo,
            synchronization=cmd.SynchronizationMetadata(node_ids, e64, e64, e64),
            dependencies=cmd.DependencyMetadata(e64, e64, e64),
            prefetch=cmd.PrefetchPlan(i64(pf_ids), i64(pf_prio), f32),
            overlap=cmd.OverlapPlan(node_ids, e64, f32), cost_model=model,
            statistics=cmd.CommunicationStatistics(
                len(local), len(remote), len(descs), 0, len(transfers), len(groups), model.total_estimated_bytes,
                model.total_estimated_latency_us, policy),
            planner_policy=policy, deterministic=getattr(cfg, "deterministic", True))


# ----------------------------------------------------------------------------- executor
def _expert_linear_weights(module: nn.Module) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(gate [I,H], up [I,H], down [H,I]) of a Qwen-style SwiGLU expert module."""
    for g, u, d in (("gate_proj", "up_proj", "down_proj"), ("w1", "w3", "w2")):
        if all(hasattr(module, n) for n in (g, u, d)):
            return (getattr(module, g).weight.detach(), getattr(module, u).weight.detach(),
                    getattr(module, d).weight.detach())
    raise ValueError("expert modules must expose gate_proj/up_proj/down_proj (or w1/w3/w2) linear layers")


class B200Executor(nn.Module):
    """Grouped tcgen05 expert GEMMs. Built from expert modules (converted once,
    like DWDP/executor/fp8.py:17-51) or from a ready ExpertWeightStore."""

    def __init__(self, config: ExecutorConfig,
                 experts: ExpertWeightStore | Mapping[int, nn.Module] | Sequence[nn.Module] | nn.Module) -> None:
        super().__init__()
        self.config = config
        if hasattr(experts, "group") and hasattr(experts, "intermediate_size"):
            self.store = experts
        else:
            if isinstance(experts, Mapping):
                mods = [experts[k] for k in sorted(experts)]
            elif isinstance(experts, nn.Module) and hasattr(experts, "expert_ids"):
                mods = [experts.get(e) for e in experts.expert_ids]  # the reference's ExpertRegistry
            else:
                mods = list(experts)
            ws = [_expert_linear_weights(m) for m in mods]
            I, H = ws[0][0].shape
            dev = ws[0][0].device if ws[0][0].is_cuda else torch.device("cuda")
            self.store = ExpertWeightStore(len(ws), H, I, weight_dtype=getattr(config, "weight_dtype", torch.float8_e4m3fn),
                                           scale_mode=getattr(config, "scale_mode", _lib.SCALE_CHANNEL), device=dev)
            for e, (g, u, d) in enumerate(ws):
                self.store.load_expert(e, g, u, d)
        self._group = self.store.group()
        self._ws: dict[tuple, torch.Tensor] = {}
        self._tl_ws = None

    def forward(self, hidden_states: torch.Tensor, dispatch_plan: DispatchPlan, execution_plan: ExecutionPlan,
                communication_plan: CommunicationPlan | None = None, workspace=None) -> ExecutorOutput:
        md = dispatch_plan.metadata
        H = self.store.hidden_size
        x = hidden_states.reshape(-1, H)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        x = x.contiguous()
        # without a gathered copy the kernels read hidden through packed_token_indices
        packed = getattr(dispatch_plan, "packed_hidden", None)
        T, K = md.num_tokens, md.top_k
        key = (T, K)
        if key not in self._ws:
            self._ws[key] = torch.empty(ops.moe_workspace_bytes(T, K, self.store.num_experts,
                                                                self.store.intermediate_size, 0),
                                        dtype=torch.uint8, device=x.device)
        w = dispatch_plan.assignments.packed_routing_weights
        if w.dtype != torch.float32:
            w = w.float()
        weighted = torch.empty(md.num_assignments, H, dtype=torch.bfloat16, device=x.device)
        if getattr(self.config, "use_tensor_list", False):
            from .tensor_list import TensorList, TensorListWorkspace, grouped_moe

            if self._tl_ws is None:
                self._tl_ws = TensorListWorkspace(x.device)
            tl = TensorList.from_plans(x, dispatch_plan, execution_plan, self._tl_ws, self.store, None, weighted,
                                       None, sync=False)
            tkey = ("tl", T, K, tl.capacity)
            if tkey not in self._ws:
                self._ws[tkey] = torch.empty(ops.moe_workspace_bytes(T, K, tl.capacity,
                                                                     self.store.intermediate_size, 0),
                                             dtype=torch.uint8, device=x.device)
            grouped_moe(tl, x, dispatch_plan, weighted, self._ws[tkey], top_k=K)
        else:
            ops.moe_experts(self._group, None, packed, x, K, md.expert_counts, md.expert_offsets, w, None,
                            weighted, None, self._ws[key],
                            packed_token_indices=dispatch_plan.assignments.packed_token_indices)
        asg = dispatch_plan.assignments
        counts, E = md.expert_counts, self.store.num_experts

        def stats() -> dict:  # DWDP/executor/outputs.py ExecutionStatistics, read on demand
            n = int((counts > 0).sum())
            return dict(num_executed_experts=n, num_skipped_experts=E - n, num_input_tokens=T,
                        num_assignments=md.num_assignments, hidden_size=H, output_size=H,
                        backend=self.config.backend)

        cp = communication_plan
        return ExecutorOutput(
            packed_expert_outputs=None, weighted_expert_outputs=weighted, expert_outputs=(),
            output_metadata=OutputMetadata(
                packed_token_indices=asg.packed_token_indices, packed_expert_ids=asg.expert_ids,
                packed_routing_weights=asg.packed_routing_weights, token_permutation=md.token_permutation,
                inverse_permutation=md.inverse_permutation, token_shape=tuple(md.token_shape), top_k=K),
            execution_metadata=ExecutionMetadata(
                execution_order=execution_plan.execution_order, expert_queue=execution_plan.expert_queue,
                expert_starts=execution_plan.expert_starts, expert_ends=execution_plan.expert_ends,
                stream_assignments=execution_plan.stream_assignments,
                communication_remote_expert_ids=cp.remote_expert_ids if cp is not None
                else torch.empty(0, dtype=torch.int64, device=x.device),
                communication_policy=cp.planner_policy if cp is not None else "static",
                scheduling_policy=execution_plan.scheduling_policy),
            statistics=LazyStatistics(stats, EXECUTION_STATISTICS_FIELDS), timing=TimingMetadata(),
            workspace=WorkspaceMetadata(used_workspace=True, workspace_bytes=int(self._ws[key].numel())),
            backend=self.config.backend, deterministic=True)


# ----------------------------------------------------------------------------- merger
class B200Merger(nn.Module):
    """Deterministic token-major merge; the output is a fresh tensor, never a workspace."""

    def __init__(self, config: MergerConfig | None = None) -> None:
        super().__init__()
        self.config = config or MergerConfig()

    def forward(self, executor_output: ExecutorOutput, workspace=None) -> MergerOutput:
        if self.config.apply_routing_weights:
            raise ValueError("the B200 executor already applies routing weights; use apply_routing_weights=False")
        if executor_output.merged_expert_outputs is not None:
            out = executor_output.merged_expert_outputs
        else:
            src = executor_output.weighted_expert_outputs
            if src is None:
                raise ValueError("executor did not provide weighted expert outputs")
            om = executor_output.output_metadata  # the reference's ExecutorOutput carries the same
            T = 1
            for s in om.token_shape:
                T *= s
            out = ops.merge(src, om.inverse_permutation, T, om.top_k,
                            out_dtype=getattr(self.config, "out_dtype", torch.bfloat16))
        H = out.shape[-1]
        om = executor_output.output_metadata
        T = out.shape[0]
        K = om.top_k
        return MergerOutput(
            hidden_states=out.reshape(*om.token_shape, H).contiguous(),
            metadata=MergeMetadata(token_shape=tuple(om.token_shape), assignment_shape=(T, K),
                                   inverse_permutation=om.inverse_permutation, top_k=K, deterministic=True),
            statistics=MergeStatistics(num_tokens=T, num_assignments=T * K, top_k=K, output_size=H,
                                       used_weighted_executor_outputs=True, backend=self.config.backend),
            timing=TimingMetadata(), workspace=WorkspaceMetadata(used_workspace=False, workspace_bytes=0),
            backend=self.config.backend, deterministic=True)


# ----------------------------------------------------------------------------- runtime
@dataclass(slots=True)
class RuntimePipelineOutput:
    """DWDP/runtime/pipeline.py:15-31: the final hidden states and every plan."""

    hidden_states: torch.Tensor
    router_output: RouterOutput
    dispatch_plan: DispatchPlan
    execution_plan: ExecutionPlan
    communication_plan: CommunicationPlan
    executor_output: ExecutorOutput
    merger_output: MergerOutput


class B200Runtime(nn.Module):
    """The six stages chained (DWDP/runtime/runtime.py:189-275)."""

    def __init__(self, router, dispatcher, scheduler, comms_planner, executor, merger) -> None:
        super().__init__()
        self.router, self.dispatcher, self.scheduler = router, dispatcher, scheduler
        self.comms_planner, self.executor, self.merger = comms_planner, executor, merger

    @classmethod
    def build_reference(cls, *, hidden_size: int, num_experts: int, top_k: int, experts,
                        router: nn.Module | None = None, executor_config: ExecutorConfig | None = None,
                        router_config: RouterConfig | None = None) -> "B200Runtime":
        router = router or B200LinearTopKRouter(router_config or RouterConfig(hidden_size, num_experts, top_k))
        return cls(router, B200ExpertMajorDispatcher(DispatcherConfig(num_experts)),
                   B200RoundRobinScheduler(SchedulerConfig()), StaticCommunicationPlanner(),
                   B200Executor(executor_config or ExecutorConfig(), experts), B200Merger())

    def forward(self, hidden_states: torch.Tensor) -> RuntimePipelineOutput:
        x = hidden_states if hidden_states.dtype == torch.bfloat16 else hidden_states.to(torch.bfloat16)
        ro = self.router(x)
        dp = self.dispatcher(ro, hidden_states=x)
        ep = self.scheduler(dp)
        cp = self.comms_planner(ep, num_experts=dp.metadata.num_experts)
        eo = self.executor(x, dp, ep, cp)
        mo = self.merger(eo)
        return RuntimePipelineOutput(mo.hidden_states, ro, dp, ep, cp, eo, mo)


register_router("b200_linear_topk", B200LinearTopKRouter)
register_dispatcher("b200_expert_major", B200ExpertMajorDispatcher)
register_scheduler("b200_round_robin", B200RoundRobinScheduler)
register_communication_planner("static", StaticCommunicationPlanner)
register_communication_planner("dwdp", DWDPCommunicationPlanner)
register_executor("b200", B200Executor)
register_merger("b200", B200Merger)


def build_router(config: RouterConfig):
    return _lookup("router", config.router_type)(config)


def build_dispatcher(config: DispatcherConfig):
    return _lookup("dispatcher", config.dispatcher_type)(config)


def build_scheduler(config: SchedulerConfig):
    return _lookup("scheduler", config.scheduling_policy)(config)


def build_executor(config: ExecutorConfig, experts):
    return _lookup("executor", config.backend)(config, experts)


def build_merger(config: MergerConfig):
    return _lookup("merger", config.backend)(config)

"""DWDP: expert weights sharded across the GPUs of one box, remote experts
prefetched over NVLink into local staging before the layer's grouped GEMM.

Ownership follows the reference's expert-parallel planner
(DWDP/comms_planner/expert_parallel.py:120-122): ``owner(e) = e // ceil(E / G)``.
Each rank keeps only its own experts' slabs; remote slabs are reached through
one CUDA IPC handle per rank (the whole slab tensor, with its allocation offset;
exchanged once with ``all_gather_object`` like
DWDP/communication/distributed.py:74-95) and copied into a staging buffer by the
communication engine. The layer's pointer arrays for staging buffer ``b`` point
at local slabs for owned experts and at staging slots for the others.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, ops
from .communication import CommunicationEngine, export_ipc_handle
from .weights import ExpertWeightStore, act_quant_code


def owner_of(expert_id: int, num_experts: int, world_size: int) -> int:
    return expert_id // math.ceil(num_experts / world_size)


def owned_experts(rank: int, num_experts: int, world_size: int) -> list[int]:
    return [e for e in range(num_experts) if owner_of(e, num_experts, world_size) == rank]


@dataclass
class ShardRecord:
    """What a rank publishes about its shard (pickled by all_gather_object)."""

    rank: int
    device: int
    owned: list[int]
    slab_bytes: int
    ipc_blob: bytes | None  # None when the shard is empty


def exchange_shard_records(record: ShardRecord, group=None) -> list[ShardRecord]:
    """All ranks' records, ordered by rank (works on any torch.distributed backend)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return [record]
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, record, group=group)
    return sorted(out, key=lambda r: r.rank)


class ShardedExpertStore:
    """E experts of one layer sharded over ``world_size`` ranks. Exposes the same
    attributes the MoE layer reads from an ExpertWeightStore (``num_experts``,
    ``hidden_size``, ``intermediate_size``, ``group()``), with ``group()``
    resolving remote experts to the currently selected staging buffer."""

    def __init__(
        self,
        num_experts: int,
        hidden_size: int,
        intermediate_size: int,
        *,
        rank: int,
        world_size: int,
        weight_dtype: torch.dtype = torch.float8_e4m3fn,
        scale_mode: int = _lib.SCALE_CHANNEL,
        device: torch.device | str = "cuda",
        num_buffers: int = 1,
        activation_quant: str = "hilo",
    ) -> None:
        self.num_experts = num_experts
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.rank = rank
        self.world_size = world_size
        self.device = torch.device(device)
        self.owned = owned_experts(rank, num_experts, world_size)
        self.local_index = {e: i for i, e in enumerate(self.owned)}
        self.local = ExpertWeightStore(max(1, len(self.owned)), hidden_size, intermediate_size,
                                       weight_dtype=weight_dtype, scale_mode=scale_mode, device=self.device,
                                       activation_quant=activation_quant)
        self.weight_dtype = self.local.weight_dtype
        self.scale_mode = self.local.scale_mode
        self.slab_bytes = self.local.slab_bytes
        self.remote = [e for e in range(num_experts) if e not in self.local_index]
        self.engine = CommunicationEngine(self.device.index or 0)
        self.engine.initialize(self.slab_bytes, len(self.remote), num_buffers)
        self.num_buffers = num_buffers
        self.buffer = 0
        self._ptrs: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]] = []
        self.records: list[ShardRecord] = []

    # ------------------------------------------------------------------ loading
    def load_expert(self, e: int, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> None:
        """Quantise/tile expert ``e`` if this rank owns it (no-op otherwise)."""
        if e in self.local_index:
            self.local.load_expert(self.local_index[e], gate, up, down)

    def nbytes_per_expert(self) -> int:
        return self.local.nbytes_per_expert()

    # ------------------------------------------------------------------ exchange
    def connect(self, group=None) -> None:
        """Publish this shard, open every other rank's shard, build the pointer
        arrays of each staging buffer. Collective over ``group``."""
        blob = export_ipc_handle(self.local.slabs) if self.owned else None
        mine = ShardRecord(self.rank, self.device.index or 0, list(self.owned), self.slab_bytes, blob)
        self.records = exchange_shard_records(mine, group)
        for e in self.owned:
            self.engine.register_expert(e, self.local.local_slab_ptr(self.local_index[e]), self.slab_bytes)
        for rec in self.records:
            if rec.rank == self.rank:
                continue
            if rec.slab_bytes != self.slab_bytes:
                raise ValueError("ranks disagree on the expert slab layout")
            for i, e in enumerate(rec.owned):
                self.engine.register_ipc_expert(e, rec.ipc_blob, self.slab_bytes, owner_device=rec.device,
                                                extra_offset=i * self.slab_bytes)
        self._build_pointer_arrays()

    def connect_local_peers(self, peers: list["ShardedExpertStore"]) -> None:
        """Single-process variant (several devices in one process): register the
        other shards by direct peer pointers instead of IPC."""
        for e in self.owned:
            self.engine.register_expert(e, self.local.local_slab_ptr(self.local_index[e]), self.slab_bytes)
        for p in peers:
            if p is self:
                continue
            for e in p.owned:
                self.engine.register_peer_expert(e, p.local.local_slab_ptr(p.local_index[e]), self.slab_bytes,
                                                 p.device.index or 0)
        self._build_pointer_arrays()

    def _build_pointer_arrays(self) -> None:
        self._ptrs = []
        for b in range(self.num_buffers):
            slabs = [self.engine.get_resident_pointer(e, b) for e in range(self.num_experts)]
            vals = self.local._pointer_values(slabs)
            self._ptrs.append(tuple(v.to(self.device) for v in vals))

    # ------------------------------------------------------------------ runtime
    def prefetch(self, buffer: int = 0) -> None:
        """Copy every remote expert into ``buffer`` (after the work already queued
        on the current stream), on the engine's copy stream."""
        self.engine.prefetch_into(self.remote, buffer)

    def wait(self, buffer: int = 0) -> None:
        self.engine.wait_buffer(buffer)

    def select_buffer(self, buffer: int) -> None:
        self.buffer = buffer

    def group(self, activation_quant: str | None = None) -> _lib.ExpertGroup:
        if not self._ptrs:
            raise RuntimeError("ShardedExpertStore.connect() has not run")
        w13, w2, s13, s2 = self._ptrs[self.buffer]
        g = _lib.ExpertGroup()
        g.act_quant = act_quant_code(activation_quant or self.local.activation_quant)
        g.num_experts = self.num_experts
        g.hidden_size = self.hidden_size
        g.intermediate_size = self.intermediate_size
        g.weight_dtype = ops.dtype_code(self.weight_dtype)
        g.scale_mode = self.scale_mode
        g.w13, g.w2, g.s13, g.s2 = w13.data_ptr(), w2.data_ptr(), s13.data_ptr(), s2.data_ptr()
        return g

    def remote_bytes(self) -> int:
        return len(self.remote) * self.nbytes_per_expert()

    def shutdown(self) -> None:
        self.engine.shutdown()

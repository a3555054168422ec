"""Expert-parallel (EP) decode path: below a batch-size threshold the token rows cross
NVLink to the rank that owns their expert, instead of every remote expert's weights
crossing to every rank (DWDP).

Mirrors the reference's hybrid switch (``DWDP/adapters/qwen15_moe.py:325-337``: EP when
``T <= ep_batch_size_threshold`` (64, ``DWDP/runtime/config.py:31``) and world > 1) and its
EP forward (``qwen15_moe.py:164-243``). The reference's four ``all_to_all_single`` calls,
host ``.tolist()`` and Python loop over local experts become, per layer, this library's
launches on one stream (no host synchronisation, graph-capturable):

    router -> ep_dispatch (peer stores) -> ep_plan + gather (owner) -> grouped e4m3 GEMMs
    (local experts + the replicated shared expert) -> ep_combine (peer stores back, wait)
    -> merge of the returned rows in slot order (+ shared expert).

The shared expert and its gate are computed where the token lives, as in the reference
(``_add_shared_expert`` after the EP forward).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib, ops
from .communication import export_ipc_handle, split_ipc_handle
from .weights import ExpertWeightStore

EP_BATCH_SIZE_THRESHOLD = 64


def ep_owner(expert_id: int, num_experts: int, world_size: int) -> int:
    """The reference's EP owner: min(e // ceil(E / world), world - 1)."""
    return min(expert_id // max(1, math.ceil(num_experts / world_size)), world_size - 1)


def ep_owned_range(rank: int, num_experts: int, world_size: int) -> tuple[int, int]:
    per = max(1, math.ceil(num_experts / world_size))
    lo = min(rank * per, num_experts)
    hi = num_experts if rank == world_size - 1 else min(num_experts, (rank + 1) * per)
    return lo, hi


def _align_up(x: int, a: int = 2 << 20) -> int:
    return (x + a - 1) // a * a


class EPExchange:
    """This rank's EP buffer, opened by every other rank through CUDA IPC. One exchange
    serves every layer of a process (layers run one after another on one stream).
    ``capacity`` = rows one rank may send to one owner = max_tokens * top_k."""

    def __init__(self, world: int, rank: int, hidden_size: int, max_tokens: int, top_k: int, device):
        if not 1 <= world <= 8:
            raise ValueError("EP supports 1..8 ranks")
        self.world, self.rank, self.H = world, rank, hidden_size
        self.max_tokens, self.top_k = max_tokens, top_k
        self.capacity = max_tokens * top_k
        self.device = torch.device(device)
        lib = _lib.load()
        nbytes = int(lib.dwdp_ep_buffer_bytes(world, hidden_size, self.capacity))
        if nbytes == 0:
            raise ValueError("bad EP buffer geometry")
        # its own allocation (2 MiB multiple) so that the IPC handle maps only this buffer
        self.buffer = torch.zeros(_align_up(nbytes), dtype=torch.uint8, device=self.device)
        self.ret_offset = int(lib.dwdp_ep_ret_offset(world, hidden_size, self.capacity))
        self._opened: list[int] = []
        self.peers = torch.zeros(world, dtype=torch.int64, device=self.device)
        self.peers[rank] = self.buffer.data_ptr()

    def connect(self, group=None) -> None:
        """Collective: publish this buffer's IPC handle, open every other rank's."""
        import torch.distributed as dist

        if self.world == 1:
            return
        blobs: list = [None] * self.world
        dist.all_gather_object(blobs, export_ipc_handle(self.buffer), group=group)
        lib = _lib.load()
        ptrs = [0] * self.world
        for r, blob in enumerate(blobs):
            if r == self.rank:
                ptrs[r] = self.buffer.data_ptr()
                continue
            handle, off = split_ipc_handle(blob)
            base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
            rc = lib.dwdp_ipc_open(handle, off, ctypes.byref(base), ctypes.byref(ptr))
            _lib.check(rc, "ipc_open", engine=True)
            self._opened.append(base.value)
            ptrs[r] = ptr.value
        self.peers.copy_(torch.tensor(ptrs, dtype=torch.int64))

    def connect_local(self, exchanges: list["EPExchange"]) -> None:
        """Single-process variant (several devices in one process, peer access enabled)."""
        self.peers.copy_(torch.tensor([ex.buffer.data_ptr() for ex in exchanges], dtype=torch.int64))

    def returned_rows(self, num_slots: int) -> torch.Tensor:
        """[num_slots, H] bf16 view of the results returned to this rank (slot order)."""
        return self.buffer[self.ret_offset: self.ret_offset + num_slots * self.H * 2].view(torch.bfloat16).view(
            num_slots, self.H)

    def close(self) -> None:
        lib = _lib.load()
        for base in self._opened:
            lib.dwdp_ipc_close(base)
        self._opened.clear()


class ExpertParallelMoE:
    """One MoE layer on the EP decode path. ``local_experts`` holds this rank's experts
    [lo, hi) of the reference's owner map in order; the shared expert is replicated."""

    def __init__(self, router_weight: torch.Tensor, local_experts: ExpertWeightStore, top_k: int,
                 exchange: EPExchange, *, shared_expert: ExpertWeightStore | None = None,
                 shared_gate_weight: torch.Tensor | None = None, router_bias: torch.Tensor | None = None,
                 renormalize: int | bool = True, eps: float = 1e-9) -> None:
        E, H = router_weight.shape
        lo, hi = ep_owned_range(exchange.rank, E, exchange.world)
        if local_experts.num_experts != max(1, hi - lo) or local_experts.hidden_size != H:
            raise ValueError(f"rank {exchange.rank} owns experts [{lo}, {hi}); the local store disagrees")
        if top_k != exchange.top_k or H != exchange.H:
            raise ValueError("exchange geometry disagrees with the layer")
        self.router_weight = router_weight.contiguous()
        self.router_bias = router_bias
        self.local = local_experts
        self.shared_expert = shared_expert
        self.shared_gate_weight = shared_gate_weight
        self.top_k, self.num_experts, self.hidden_size = top_k, E, H
        self.renormalize, self.eps = renormalize, eps
        self.fused_routing = True  # as MoELayer: one-launch router + dispatch at the smallest sizes
        self.ex = exchange
        self.lo, self.hi = lo, hi
        self._routed_group = local_experts.group()
        self._shared_group = shared_expert.group(local_experts.activation_quant) if shared_expert is not None else None
        self._ws: dict[int, dict] = {}

    def workspace(self, T: int) -> dict:
        ws = self._ws.get(T)
        if ws is not None:
            return ws
        if T > self.ex.max_tokens:
            raise ValueError(f"EP path takes at most {self.ex.max_tokens} tokens per rank")
        ex, K, E, H, dev = self.ex, self.top_k, self.num_experts, self.hidden_size, self.ex.device
        El = self.local.num_experts
        # Rows this rank may receive as an owner: up to `capacity` from every source, whatever
        # this rank's own T is (ranks may run different token counts, T = 0 included), so the
        # owner's expert GEMMs are sized for world * capacity rows.
        cap_rows = ex.world * ex.capacity
        Is = self.shared_expert.intermediate_size if self.shared_expert is not None else 0
        parts = ops.moe_shared_parts(T, Is) if self.shared_expert is not None else 0
        ws = dict(
            router=ops.RouterResult(
                router_logits=torch.empty(T, E, dtype=torch.float32, device=dev),
                routing_probabilities=torch.empty(T, K, dtype=torch.float32, device=dev),
                topk_indices=torch.empty(T, K, dtype=torch.int64, device=dev),
                topk_weights=torch.empty(T, K, dtype=torch.float32, device=dev),
                shared_gate=torch.empty(T, dtype=torch.float32, device=dev)
                if (self.shared_expert is not None and self.shared_gate_weight is not None) else None),
            counts=torch.zeros(El, dtype=torch.int64, device=dev),
            offsets=torch.zeros(El + 1, dtype=torch.int64, device=dev),
            packed_src=torch.zeros(cap_rows, dtype=torch.int32, device=dev),
            packed_w=torch.zeros(cap_rows, dtype=torch.float32, device=dev),
            ret_addr=torch.zeros(cap_rows, dtype=torch.int32, device=dev),
            total=torch.zeros(1, dtype=torch.int32, device=dev),
            packed_hidden=torch.zeros(cap_rows, H, dtype=torch.bfloat16, device=dev),
            weighted=torch.empty(cap_rows, H, dtype=torch.bfloat16, device=dev),
            shared_out=torch.empty(parts, T, H, dtype=torch.bfloat16, device=dev) if parts else None,
            parts=parts,
            moe_ws=torch.empty(ops.moe_workspace_bytes(cap_rows, 1, El, self.local.intermediate_size, 0),
                               dtype=torch.uint8, device=dev),
            shared_ws=torch.empty(ops.moe_shared_workspace_bytes(T, H, Is), dtype=torch.uint8, device=dev)
            if parts else None,
            inv=torch.arange(T * K, dtype=torch.int64, device=dev),
            # the one-launch router + dispatch of MoELayer at the smallest sizes (its dispatch
            # outputs are not used here; the same routing kernel keeps EP bit-identical to it)
            fdisp=ops.DispatchResult(*(torch.empty(n, dtype=torch.int64, device=dev)
                                       for n in (E, E + 1, T * K, T * K, T * K, T * K)),
                                     torch.empty(T * K, dtype=torch.float32, device=dev), None),
            ticket=torch.zeros(1, dtype=torch.int32, device=dev),
            gate_logit=torch.empty(max(T, 1), dtype=torch.float32, device=dev),
            status=torch.zeros(4, dtype=torch.int32, device=dev),
        )
        self._ws[T] = ws
        return ws

    def forward(self, x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.dtype != torch.bfloat16 or x.shape[-1] != self.hidden_size:
            raise ValueError("EP layer expects bf16 [T, H] hidden states")
        x = x.reshape(-1, self.hidden_size).contiguous()
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        # T == 0 still runs the exchange: this rank owns experts other ranks' tokens may pick,
        # and every rank's arrival counters must advance once per layer
        self.run(x, self.workspace(T), out)
        return out

    __call__ = forward

    def run(self, x: torch.Tensor, ws: dict, out: torch.Tensor) -> None:
        ex, K, T, H = self.ex, self.top_k, x.shape[0], self.hidden_size
        lib, stream = _lib.load(), torch.cuda.current_stream().cuda_stream
        r = ws["router"]
        gate_w = self.shared_gate_weight if self.shared_expert is not None else None
        if self.fused_routing and T > 0 and ops.use_fused_routing(T, K, self.num_experts, x, self.router_weight):
            ops.route_dispatch_small(x, self.router_weight, K, r, ws["fdisp"], ws["ticket"], ws["gate_logit"],
                                     bias=self.router_bias, shared_gate_weight=gate_w, renormalize=self.renormalize,
                                     eps=self.eps, status=ws["status"])
        else:
            ops.router_topk(x, self.router_weight, K, bias=self.router_bias, shared_gate_weight=gate_w,
                            renormalize=self.renormalize, eps=self.eps, out=r)
        st = ws["status"].data_ptr()
        rc = lib.dwdp_ep_dispatch(x.data_ptr(), r.topk_indices.data_ptr(), r.topk_weights.data_ptr(), T, K,
                                  self.num_experts, ex.world, ex.rank, H, ex.capacity, ex.peers.data_ptr(), st,
                                  stream)
        _lib.check(rc, "ep_dispatch")
        rc = lib.dwdp_ep_plan(ex.buffer.data_ptr(), ex.world, ex.rank, H, ex.capacity, self.num_experts, self.lo,
                              self.local.num_experts, ws["counts"].data_ptr(), ws["offsets"].data_ptr(),
                              ws["packed_src"].data_ptr(), ws["packed_w"].data_ptr(), ws["ret_addr"].data_ptr(),
                              ws["total"].data_ptr(), ws["packed_hidden"].data_ptr(), st, stream)
        _lib.check(rc, "ep_plan")
        # received rows: sized for every source's full capacity (counts/offsets pick the real ones)
        ops.moe_experts(self._routed_group, None, ws["packed_hidden"], ws["packed_hidden"], 1, ws["counts"],
                        ws["offsets"], ws["packed_w"], None, ws["weighted"], None, ws["moe_ws"], ws["status"])
        rc = lib.dwdp_ep_combine(ex.buffer.data_ptr(), ex.world, ex.rank, H, ex.capacity, ws["weighted"].data_ptr(),
                                 ws["ret_addr"].data_ptr(), ws["total"].data_ptr(), ex.peers.data_ptr(), st, stream)
        _lib.check(rc, "ep_combine")
        if T == 0:
            return
        if self.shared_expert is not None:
            # the shared expert over this rank's own tokens, gated in its down epilogue as in
            # MoELayer's grouped launch (bit-identical partials), then the merge
            ops.moe_shared_expert(self._shared_group, x, ws["shared_out"], ws["shared_ws"], ws["status"],
                                  shared_gate=r.shared_gate)
            ops.merge(ex.returned_rows(T * K), ws["inv"], T, K, shared_out=ws["shared_out"],
                      shared_parts=ws["parts"], out=out)
        else:
            ops.merge(ex.returned_rows(T * K), ws["inv"], T, K, out=out)

    def read_status(self, T: int) -> tuple[int, ...]:
        return tuple(self.workspace(T)["status"].cpu().tolist())

    def kernel_launches(self) -> int:
        """router, ep_send, ep_plan, ep_gather, the received rows' expert GEMMs (plan+planes,
        gate/up, [planes,] down), ep_return, ep_wait, the shared expert's own GEMMs, merge."""
        gemm = 3 if self.local.activation_quant == "block128" else 4
        return 4 + gemm + 2 + (gemm if self.shared_expert is not None else 0) + 1

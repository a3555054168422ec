"""Full Qwen1.5-MoE decode step: the model around the MoE layers, over a paged KV cache,
captured as ONE CUDA graph per batch size.

What the reference does for this step: its HF adapter swaps each Qwen2-MoE sparse block
for a DWDP block and leaves the HF decoder around it (``DWDP/adapters/qwen15_moe.py:
434-580``). Graph capture is per MoE block and lazy per input shape
(``qwen15_moe.py:285-300``, ``DWDP/runtime/cuda_graph.py:63-201``). The KV cache
manager is a free list over fixed-size blocks (``DWDP/runtime/paged_attention.py:20-76``).

Here the whole step is one graph: embedding gather, then per layer
``add_rmsnorm -> qkv GEMM -> rope_append_kv -> paged_attention -> o GEMM ->
add_rmsnorm -> MoELayer.run``, then the final norm and the lm_head GEMM. The dense
projections are plain cuBLAS GEMMs; everything else is this library's kernels. The
cache keeps each layer's K and V pages contiguous ([L, 2, blocks, block_size, NH, D]
instead of the reference's [blocks, L, 2, ...]), so one layer's attention reads one
region of HBM.
"""
from __future__ import annotations

import collections
from dataclasses import dataclass

import torch

from . import _lib, ops
from .layer import MoELayer
from .weights import ExpertWeightStore


@dataclass(frozen=True)
class QwenMoEConfig:
    """Qwen1.5-MoE-A2.7B shapes (hidden 2048, 24 layers, 16 heads of 128, 60 experts of
    1408, top-4, shared expert 5632 with a sigmoid gate, rope theta 1e6, vocab 151936)."""

    vocab_size: int = 151936
    hidden_size: int = 2048
    num_layers: int = 24
    num_heads: int = 16
    head_dim: int = 128
    num_experts: int = 60
    moe_intermediate_size: int = 1408
    top_k: int = 4
    shared_intermediate_size: int = 5632
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    block_size: int = 16
    max_context: int = 2048


class PagedKVCacheManager:
    """Free-list block manager with the reference's interface (``allocate`` pops the
    lowest free ids, raising ``RuntimeError`` when the pool is short; ``free`` drops a
    reference and returns the block at zero), DWDP/runtime/paged_attention.py:20-76.
    Storage: ``kv_cache[layer, 0|1]`` is that layer's K|V page array
    [num_blocks, block_size, num_heads, head_dim]."""

    def __init__(self, num_blocks: int, block_size: int = 16, num_layers: int = 32, num_heads: int = 32,
                 head_dim: int = 128, dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda"):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.free_blocks: collections.deque[int] = collections.deque(range(num_blocks))
        self.ref_counts: dict[int, int] = {}
        self.kv_cache = torch.empty(num_layers, 2, num_blocks, block_size, num_heads, head_dim, dtype=dtype,
                                    device=self.device)

    @property
    def used_blocks(self) -> dict[int, int]:
        return self.ref_counts

    def allocate(self, num_needed_blocks: int) -> list[int]:
        if len(self.free_blocks) < num_needed_blocks:
            raise RuntimeError(f"Out of KV Cache memory: requested {num_needed_blocks} blocks, but only "
                               f"{len(self.free_blocks)} available.")
        out = [self.free_blocks.popleft() for _ in range(num_needed_blocks)]
        for b in out:
            self.ref_counts[b] = 1
        return out

    def free(self, block_ids: list[int]) -> None:
        for b in block_ids:
            if b in self.ref_counts:
                self.ref_counts[b] -= 1
                if self.ref_counts[b] <= 0:
                    del self.ref_counts[b]
                    self.free_blocks.append(b)

    def k(self, layer: int) -> torch.Tensor:
        return self.kv_cache[layer, 0]

    def v(self, layer: int) -> torch.Tensor:
        return self.kv_cache[layer, 1]


@dataclass
class AttentionWeights:
    input_norm: torch.Tensor  # [H] bf16
    wqkv: torch.Tensor  # [3H, H] bf16 (q | k | v rows)
    bqkv: torch.Tensor  # [3H] bf16
    wo: torch.Tensor  # [H, H] bf16
    post_norm: torch.Tensor  # [H] bf16


def random_moe_layer(cfg: QwenMoEConfig, device, seed: int) -> MoELayer:
    """Random-init MoE block: router W ~ N(0, 1/H), experts and shared expert ~ N(0, 0.02)
    quantised to e4m3 with per-output-channel scales, shared gate ~ N(0, 0.02)."""
    H, E, I, Is = cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_intermediate_size
    g = torch.Generator(device=device).manual_seed(seed)
    wr = (torch.randn(E, H, generator=g, device=device) / H**0.5).bfloat16()
    store = ExpertWeightStore(E, H, I, weight_dtype=torch.float8_e4m3fn, scale_mode=_lib.SCALE_CHANNEL, device=device)
    for e in range(E):
        store.load_expert(e, torch.randn(I, H, generator=g, device=device) * 0.02,
                          torch.randn(I, H, generator=g, device=device) * 0.02,
                          torch.randn(H, I, generator=g, device=device) * 0.02)
    shared = ExpertWeightStore(1, H, Is, weight_dtype=torch.float8_e4m3fn, scale_mode=_lib.SCALE_CHANNEL,
                               device=device)
    shared.load_expert(0, torch.randn(Is, H, generator=g, device=device) * 0.02,
                       torch.randn(Is, H, generator=g, device=device) * 0.02,
                       torch.randn(H, Is, generator=g, device=device) * 0.02)
    gate = (torch.randn(H, generator=g, device=device) * 0.02).bfloat16()
    return MoELayer(wr, store, cfg.top_k, shared_expert=shared, shared_gate_weight=gate)


@dataclass
class _StepBuffers:
    B: int
    tokens: torch.Tensor  # [B] int64
    positions: torch.Tensor  # [B] int32
    seq_lens: torch.Tensor  # [B] int32
    block_table: torch.Tensor  # [B, max_blocks] int32
    h: torch.Tensor  # residual stream [B, H]
    xn: torch.Tensor  # normed rows [B, H]
    qkv: torch.Tensor  # [B, 3H]
    q: torch.Tensor  # [B, NH, D]
    attn: torch.Tensor  # [B, NH, D]
    delta: torch.Tensor  # o_proj / MoE output [B, H]
    logits: torch.Tensor  # [B, V]
    next_tokens: torch.Tensor  # [B] int64
    attn_ws: torch.Tensor
    splits: int
    status: torch.Tensor  # [4] int32
    moe_ws: list
    graph: torch.cuda.CUDAGraph | None = None
    moe_graph: torch.cuda.CUDAGraph | None = None


class QwenMoEDecodeModel:
    """Random-init Qwen1.5-MoE-shaped decoder (synthetic weights; no checkpoint is
    loaded) whose decode step runs as one CUDA graph per batch size."""

    def __init__(self, cfg: QwenMoEConfig, device, *, seed: int = 1235, num_blocks: int | None = None,
                 max_batch: int = 1):
        self.cfg = cfg
        self.device = torch.device(device)
        H, NH, D, V = cfg.hidden_size, cfg.num_heads, cfg.head_dim, cfg.vocab_size
        if NH * D != H:
            raise ValueError("num_heads * head_dim must equal hidden_size")
        g = torch.Generator(device=device).manual_seed(seed)

        def rn(*shape, std=0.02):
            return (torch.randn(*shape, generator=g, device=device) * std).bfloat16()

        self.embed = rn(V, H)
        self.attn: list[AttentionWeights] = []
        for _ in range(cfg.num_layers):
            self.attn.append(AttentionWeights(
                input_norm=(1.0 + rn(H, std=0.1).float()).bfloat16(), wqkv=rn(3 * H, H), bqkv=rn(3 * H, std=0.1),
                wo=rn(H, H), post_norm=(1.0 + rn(H, std=0.1).float()).bfloat16()))
        self.moe = [random_moe_layer(cfg, device, seed + 1 + l) for l in range(cfg.num_layers)]
        self.final_norm = (1.0 + rn(H, std=0.1).float()).bfloat16()
        self.lm_head = rn(V, H)
        self.max_blocks = -(-cfg.max_context // cfg.block_size)
        self.cache = PagedKVCacheManager(num_blocks or self.max_blocks * max_batch, cfg.block_size, cfg.num_layers,
                                         NH, D, torch.bfloat16, device)
        self._bufs: dict[int, _StepBuffers] = {}

    # ------------------------------------------------------------------ sequences
    def admit(self, num_sequences: int) -> torch.Tensor:
        """Allocate max_context worth of blocks per new sequence; returns the [B, max_blocks]
        int32 block table (host)."""
        rows = [self.cache.allocate(self.max_blocks) for _ in range(num_sequences)]
        return torch.tensor(rows, dtype=torch.int32)

    def release(self, block_table: torch.Tensor) -> None:
        for row in block_table.tolist():
            self.cache.free([b for b in row if b >= 0])

    def fill_context(self, seed: int = 7) -> None:
        """Synthetic prior context: every K/V page ~ N(0, 1)."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        for l in range(self.cfg.num_layers):
            self.cache.kv_cache[l].normal_(generator=g)

    # ------------------------------------------------------------------ step
    def buffers(self, B: int) -> _StepBuffers:
        b = self._bufs.get(B)
        if b is not None:
            return b
        cfg, dev = self.cfg, self.device
        H, NH, D = cfg.hidden_size, cfg.num_heads, cfg.head_dim
        splits = ops.paged_attention_splits(B, NH, cfg.max_context, cfg.block_size)
        bf = dict(dtype=torch.bfloat16, device=dev)
        b = _StepBuffers(
            B=B, tokens=torch.zeros(B, dtype=torch.int64, device=dev),
            positions=torch.zeros(B, dtype=torch.int32, device=dev),
            seq_lens=torch.ones(B, dtype=torch.int32, device=dev),
            block_table=torch.zeros(B, self.max_blocks, dtype=torch.int32, device=dev),
            h=torch.empty(B, H, **bf), xn=torch.empty(B, H, **bf), qkv=torch.empty(B, 3 * H, **bf),
            q=torch.empty(B, NH, D, **bf), attn=torch.empty(B, NH, D, **bf), delta=torch.empty(B, H, **bf),
            logits=torch.empty(B, cfg.vocab_size, **bf), next_tokens=torch.zeros(B, dtype=torch.int64, device=dev),
            attn_ws=ops.paged_attention_workspace(B, NH, splits, dev), splits=splits,
            status=torch.zeros(4, dtype=torch.int32, device=dev),
            moe_ws=[m.workspace(B) for m in self.moe])
        self._bufs[B] = b
        return b

    def _attention(self, l: int, b: _StepBuffers) -> None:
        cfg, w = self.cfg, self.attn[l]
        torch.matmul(b.xn, w.wqkv.t(), out=b.qkv)
        ops.rope_append_kv(b.qkv, w.bqkv, b.positions, b.block_table, self.cache.k(l), self.cache.v(l),
                           cfg.rope_theta, q_out=b.q, status=b.status)
        ops.paged_attention(b.q, self.cache.k(l), self.cache.v(l), b.block_table, b.seq_lens, cfg.max_context,
                            splits=b.splits, workspace=b.attn_ws, out=b.attn, status=b.status)
        torch.matmul(b.attn.view(b.B, -1), w.wo.t(), out=b.delta)

    def _step(self, b: _StepBuffers) -> None:
        cfg = self.cfg
        ops.gather_rows(self.embed, b.tokens, out=b.h)
        for l in range(cfg.num_layers):
            ops.add_rmsnorm(b.h, None if l == 0 else b.delta, self.attn[l].input_norm, cfg.rms_norm_eps, out=b.xn)
            self._attention(l, b)
            ops.add_rmsnorm(b.h, b.delta, self.attn[l].post_norm, cfg.rms_norm_eps, out=b.xn)
            self.moe[l].run(b.xn, b.moe_ws[l], b.delta)
        ops.add_rmsnorm(b.h, b.delta, self.final_norm, cfg.rms_norm_eps, out=b.xn)
        torch.matmul(b.xn, self.lm_head.t(), out=b.logits)
        torch.argmax(b.logits, dim=-1, out=b.next_tokens)

    def _moe_only(self, b: _StepBuffers) -> None:
        for l in range(self.cfg.num_layers):
            self.moe[l].run(b.xn, b.moe_ws[l], b.delta)

    def set_inputs(self, tokens: torch.Tensor, positions: torch.Tensor, block_table: torch.Tensor) -> _StepBuffers:
        """Copy one step's inputs (host or device) into the static buffers of batch size B;
        seq_lens = positions + 1 (the new token attends to itself)."""
        B = tokens.shape[0]
        b = self.buffers(B)
        if int(positions.max()) >= self.cfg.max_context or int(positions.min()) < 0:
            raise ValueError(f"positions must lie in [0, {self.cfg.max_context})")
        b.tokens.copy_(tokens, non_blocking=True)
        b.positions.copy_(positions.to(torch.int32), non_blocking=True)
        b.seq_lens.copy_((positions.to(torch.int32) + 1), non_blocking=True)
        b.block_table.copy_(block_table, non_blocking=True)
        return b

    def capture(self, B: int, warmup: int = 2) -> _StepBuffers:
        """Capture the step (and a graph of its MoE layers alone) for batch size B. Warm-up
        runs on the capture stream first, as graph capture requires; they write the KV slots
        at the current positions, which the next real step overwrites."""
        b = self.buffers(B)
        if b.graph is not None:
            return b
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._step(b)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        b.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(b.graph):
            self._step(b)
        b.moe_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(b.moe_graph):
            self._moe_only(b)
        return b

    def step(self, tokens: torch.Tensor, positions: torch.Tensor, block_table: torch.Tensor, *,
             graph: bool = True) -> torch.Tensor:
        """One decode step for B sequences: returns the [B] next-token ids (device, greedy) and
        leaves the logits in ``buffers(B).logits``."""
        b = self.set_inputs(tokens, positions, block_table)
        if graph:
            self.capture(b.B).graph.replay()
        else:
            self._step(b)
        return b.next_tokens

    def read_status(self, B: int) -> tuple[int, ...]:
        b = self.buffers(B)
        st = tuple(int(v) for v in b.status.cpu())
        for l, m in enumerate(self.moe):
            ms = m.read_status(B)
            if ms[0] != 0 and st[0] == 0:
                st = ms
        return st

    def kernel_launches(self, B: int) -> int:
        """This library's kernels per step (cuBLAS GEMMs and the argmax are not counted)."""
        per_layer = 2 + 1 + 2  # two add_rmsnorm, rope_append_kv, attention + combine
        return 1 + sum(per_layer + m.kernel_launches(B) for m in self.moe) + 1

    def kv_bytes_per_step(self, seq_lens: list[int]) -> int:
        """Algorithmic K/V bytes the attention reads in one step (every layer)."""
        per_pos = 2 * self.cfg.num_heads * self.cfg.head_dim * 2
        return self.cfg.num_layers * per_pos * sum(seq_lens)

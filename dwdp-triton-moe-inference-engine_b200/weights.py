"""Expert weight store: the device-resident form of the experts' SwiGLU weights.

Replaces the reference's weight provider + TensorList pointer arrays
(DWDP/executor/weights.py:225-315, DWDP/executor/tensor_list.py:29-67) and its
one-shot FP8 conversion (DWDP/executor/fp8.py:17-51, 118-146).

Each expert is ONE contiguous slab ``[gate/up tiles | down tiles | gate/up scales
| down scales]`` so that DWDP can move a whole expert across NVLink with a single
copy and re-point the kernel at it by rewriting one entry of each pointer array.
The pointer arrays (``w13``/``w2``/``s13``/``s2``, int64 device tensors) are what
the grouped GEMM reads, like TensorList's gate/down pointer fields.
"""
from __future__ import annotations

import torch

from . import _lib, ops


ACTIVATION_QUANT = {"hilo": _lib.ACT_HILO, "block128": _lib.ACT_BLOCK128}


def check_activation_quant(mode: str) -> str:
    if mode not in ACTIVATION_QUANT:
        raise ValueError(f"activation_quant must be one of {sorted(ACTIVATION_QUANT)}, got {mode!r}")
    return mode


def act_quant_code(mode: str) -> int:
    return ACTIVATION_QUANT[check_activation_quant(mode)]


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class ExpertWeightStore:
    """Packed weights of ``num_experts`` SwiGLU experts with hidden size H and
    intermediate size I. ``weight_dtype`` is ``torch.float8_e4m3fn`` (with
    ``scale_mode`` CHANNEL, BLOCK128 or TENSOR) or ``torch.bfloat16`` (no scale).

    ``activation_quant`` picks how the e4m3 GEMMs carry the activations:
    ``"hilo"`` (two e4m3 planes per row, about bf16 precision) or ``"block128"``
    (one e4m3 plane with one scale per (row, 128 channels), the reference's FP8
    scheme, DWDP/executor/fp8.py:86-115; the tensor core does half the work)."""

    def __init__(
        self,
        num_experts: int,
        hidden_size: int,
        intermediate_size: int,
        *,
        weight_dtype: torch.dtype = torch.float8_e4m3fn,
        scale_mode: int = _lib.SCALE_CHANNEL,
        device: torch.device | str = "cuda",
        slabs: torch.Tensor | None = None,
        activation_quant: str = "hilo",
    ) -> None:
        if hidden_size % 128 or intermediate_size % 128:
            raise ValueError("hidden_size and intermediate_size must be multiples of 128")
        if weight_dtype == torch.bfloat16:
            scale_mode = _lib.SCALE_NONE
        elif weight_dtype == torch.float8_e4m3fn:
            if scale_mode not in (_lib.SCALE_CHANNEL, _lib.SCALE_BLOCK128, _lib.SCALE_TENSOR):
                raise ValueError("fp8 weights need SCALE_CHANNEL, SCALE_BLOCK128 or SCALE_TENSOR")
        else:
            raise ValueError("weight_dtype must be torch.float8_e4m3fn or torch.bfloat16")
        self.num_experts = num_experts
        self.hidden_size = H = hidden_size
        self.intermediate_size = I = intermediate_size
        self.weight_dtype = weight_dtype
        self.scale_mode = scale_mode
        self.activation_quant = check_activation_quant(activation_quant)
        self.device = torch.device(device)
        esz = 1 if weight_dtype == torch.float8_e4m3fn else 2
        self.w13_bytes = 2 * I * H * esz
        self.w2_bytes = H * I * esz
        if weight_dtype == torch.float8_e4m3fn:
            per_row = scale_mode != _lib.SCALE_BLOCK128  # CHANNEL and TENSOR keep one scale per row
            self.s13_floats = 2 * I if per_row else 2 * (I // 128) * (H // 128)
            self.s2_floats = H if per_row else (H // 128) * (I // 128)
        else:
            self.s13_floats = self.s2_floats = 0
        self.off_w2 = _align(self.w13_bytes)
        self.off_s13 = _align(self.off_w2 + self.w2_bytes)
        self.off_s2 = _align(self.off_s13 + 4 * self.s13_floats)
        self.slab_bytes = _align(self.off_s2 + 4 * self.s2_floats, 1024)
        if slabs is None:
            slabs = torch.zeros(num_experts, self.slab_bytes, dtype=torch.uint8, device=self.device)
        elif tuple(slabs.shape) != (num_experts, self.slab_bytes) or slabs.dtype != torch.uint8:
            raise ValueError("slabs must be a uint8 [num_experts, slab_bytes] tensor")
        self.slabs = slabs
        self.w13_ptrs = torch.zeros(num_experts, dtype=torch.int64, device=self.device)
        self.w2_ptrs = torch.zeros_like(self.w13_ptrs)
        self.s13_ptrs = torch.zeros_like(self.w13_ptrs)
        self.s2_ptrs = torch.zeros_like(self.w13_ptrs)
        self.reset_pointers()

    # ------------------------------------------------------------------ pointers
    def local_slab_ptr(self, e: int) -> int:
        return self.slabs.data_ptr() + e * self.slab_bytes

    def _pointer_values(self, slab_ptrs: list[int]) -> torch.Tensor:
        has_scale = self.s13_floats > 0
        rows = [
            [p, p + self.off_w2, p + self.off_s13 if has_scale else 0, p + self.off_s2 if has_scale else 0]
            for p in slab_ptrs
        ]
        return torch.tensor(rows, dtype=torch.int64).T.contiguous()

    def reset_pointers(self) -> None:
        """Point every expert at its own slab in ``self.slabs``."""
        self.set_slab_pointers([self.local_slab_ptr(e) for e in range(self.num_experts)])

    def set_slab_pointers(self, slab_ptrs: list[int]) -> None:
        """Point expert e at the slab image starting at ``slab_ptrs[e]`` (a local
        slab, a staging buffer, ...). One H2D copy per pointer array."""
        vals = self._pointer_values(slab_ptrs)
        for dst, row in zip((self.w13_ptrs, self.w2_ptrs, self.s13_ptrs, self.s2_ptrs), vals):
            dst.copy_(row, non_blocking=False)

    # ------------------------------------------------------------------ filling
    def load_expert(self, e: int, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> None:
        """Quantise/tile one expert from nn.Linear-layout weights gate/up [I,H], down [H,I]."""
        I, H = self.intermediate_size, self.hidden_size
        if tuple(gate.shape) != (I, H) or tuple(up.shape) != (I, H) or tuple(down.shape) != (H, I):
            raise ValueError(
                f"expert {e}: expected gate/up {(I, H)} and down {(H, I)}, got "
                f"{tuple(gate.shape)}, {tuple(up.shape)}, {tuple(down.shape)}"
            )
        dev = self.device
        src_dtype = torch.float32 if gate.dtype == torch.float32 else torch.bfloat16
        g = gate.to(device=dev, dtype=src_dtype)
        u = up.to(device=dev, dtype=src_dtype)
        d = down.to(device=dev, dtype=src_dtype)
        t13, sc13 = ops.pack_weights([g, u], self.weight_dtype, self.scale_mode)
        t2, sc2 = ops.pack_weights([d], self.weight_dtype, self.scale_mode)
        s = self.slabs[e]
        s[: self.w13_bytes].copy_(t13)
        s[self.off_w2 : self.off_w2 + self.w2_bytes].copy_(t2)
        if sc13 is not None:
            s[self.off_s13 : self.off_s13 + 4 * self.s13_floats].copy_(sc13.view(torch.uint8))
            s[self.off_s2 : self.off_s2 + 4 * self.s2_floats].copy_(sc2.view(torch.uint8))

    @classmethod
    def from_weights(
        cls,
        gate: torch.Tensor,
        up: torch.Tensor,
        down: torch.Tensor,
        *,
        weight_dtype: torch.dtype = torch.float8_e4m3fn,
        scale_mode: int = _lib.SCALE_CHANNEL,
        device: torch.device | str = "cuda",
        activation_quant: str = "hilo",
    ) -> "ExpertWeightStore":
        """Build from stacked [E, I, H] gate/up and [E, H, I] down weights."""
        E, I, H = gate.shape
        store = cls(E, H, I, weight_dtype=weight_dtype, scale_mode=scale_mode, device=device,
                    activation_quant=activation_quant)
        for e in range(E):
            store.load_expert(e, gate[e], up[e], down[e])
        return store

    # ------------------------------------------------------------------ reading
    def quantized(self, e: int) -> dict[str, torch.Tensor]:
        """Raw packed sections of expert ``e`` (tiles and scales)."""
        s = self.slabs[e]
        out = {"w13": s[: self.w13_bytes], "w2": s[self.off_w2 : self.off_w2 + self.w2_bytes]}
        if self.s13_floats:
            out["s13"] = s[self.off_s13 : self.off_s13 + 4 * self.s13_floats].view(torch.float32)
            out["s2"] = s[self.off_s2 : self.off_s2 + 4 * self.s2_floats].view(torch.float32)
        return out

    def dequantized(self, e: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """fp32 (gate, up, down) exactly as the kernels see them."""
        I, H = self.intermediate_size, self.hidden_size
        q = self.quantized(e)
        w13 = ops.unpack_weights(q["w13"], q.get("s13"), I, H, 2, self.weight_dtype, self.scale_mode)
        w2 = ops.unpack_weights(q["w2"], q.get("s2"), H, I, 1, self.weight_dtype, self.scale_mode)
        return w13[0], w13[1], w2[0]

    # ------------------------------------------------------------------ handles
    def group(self, activation_quant: str | None = None) -> _lib.ExpertGroup:
        """The ``dwdp_expert_group`` handle the C ABI takes (``activation_quant``
        overrides the store's setting for this handle)."""
        g = _lib.ExpertGroup()
        g.act_quant = act_quant_code(activation_quant or self.activation_quant)
        g.num_experts = self.num_experts
        g.hidden_size = self.hidden_size
        g.intermediate_size = self.intermediate_size
        g.weight_dtype = ops.dtype_code(self.weight_dtype)
        g.scale_mode = self.scale_mode
        g.w13 = self.w13_ptrs.data_ptr()
        g.w2 = self.w2_ptrs.data_ptr()
        g.s13 = self.s13_ptrs.data_ptr()
        g.s2 = self.s2_ptrs.data_ptr()
        return g

    def nbytes_per_expert(self) -> int:
        """Bytes of one expert's weights + scales (what one use must read)."""
        return self.w13_bytes + self.w2_bytes + 4 * (self.s13_floats + self.s2_floats)

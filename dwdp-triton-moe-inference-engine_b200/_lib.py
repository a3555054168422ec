"""ctypes binding of the C-ABI library ``libdwdp_b200.so`` (include/dwdp_b200.h).

The library is loaded from this package directory. There is no fallback: if the
library is missing or fails to load, every op raises ``RuntimeError`` instead of
computing anything on the CPU.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libdwdp_b200.so"

DWDP_OK = 0
DWDP_ERR_INVALID_ARGUMENT = -1
DWDP_ERR_CAPACITY = -2
DWDP_ERR_CUDA = -3
DWDP_ERR_DEVICE_TIMEOUT = -4
DWDP_ERR_DEVICE_BOUNDS = -5
DWDP_ERR_UNSUPPORTED = -6
DWDP_ERR_STATE = -7
DWDP_ERR_NOT_FOUND = -8

DTYPE_F16 = 1
DTYPE_BF16 = 2
DTYPE_FP8_E4M3 = 3
DTYPE_F32 = 4

SCALE_NONE = 0
SCALE_CHANNEL = 1
SCALE_BLOCK128 = 2
SCALE_TENSOR = 3

ACT_HILO = 0
ACT_BLOCK128 = 1

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t


class ExpertGroup(ctypes.Structure):
    """Mirror of ``dwdp_expert_group`` (device pointer arrays per expert)."""

    _fields_ = [
        ("num_experts", c_int),
        ("hidden_size", c_int),
        ("intermediate_size", c_int),
        ("weight_dtype", c_int),
        ("scale_mode", c_int),
        ("w13", c_void_p),
        ("w2", c_void_p),
        ("s13", c_void_p),
        ("s2", c_void_p),
        ("act_quant", c_int),
    ]


TL_ROWS = 27  # DWDP_TL_ROWS: the reference's 26 TensorList fields + the down-scale row


class TensorListBases(ctypes.Structure):
    """Mirror of ``dwdp_tensor_list_bases``."""

    _fields_ = [(n, c_void_p) for n in ("input", "token_index", "routing_weights", "intermediate", "output",
                                        "weighted_output")] + [
        (n, c_int64) for n in ("intermediate_row_bytes", "output_row_bytes", "weighted_row_bytes", "n", "k",
                               "intermediate_n", "input_ld", "gate_ld", "up_ld", "down_ld", "output_ld",
                               "dtype_code")]


class TensorListHandle(ctypes.Structure):
    """Mirror of ``dwdp_tensor_list``."""

    _fields_ = [("capacity", c_int64), ("fields", c_void_p), ("hidden_size", c_int),
                ("intermediate_size", c_int), ("weight_dtype", c_int), ("scale_mode", c_int),
                ("act_quant", c_int)]


class CopySlice(ctypes.Structure):
    """Mirror of ``dwdp_copy_slice``."""

    _fields_ = [("expert_id", c_int), ("reserved", c_int), ("start", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "dwdp_version": (c_int, []),
    "dwdp_last_error": (ctypes.c_char_p, []),
    "dwdp_device_sm_count": (c_int, []),
    "dwdp_router_topk": (
        c_int,
        [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
         c_float, c_int, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p],
    ),
    "dwdp_dispatch_scratch_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "dwdp_dispatch": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
         c_void_p],
    ),
    "dwdp_dispatch_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p],
    ),
    "dwdp_dispatch_noalloc_max_scratch_bytes": (c_size_t, []),
    "dwdp_route_dispatch_small": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_float, c_int, c_float]
        + [c_void_p] * 16
    ),
    "dwdp_quantize_activations_blockwise": (
        c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p]
    ),
    "dwdp_gather_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p, c_void_p, c_void_p]),
    "dwdp_ep_buffer_bytes": (c_size_t, [c_int, c_int, c_int]),
    "dwdp_ep_ret_offset": (c_size_t, [c_int, c_int, c_int]),
    "dwdp_ipc_open": (c_int, [c_void_p, c_size_t, c_void_p, c_void_p]),
    "dwdp_ipc_close": (c_int, [c_void_p]),
    "dwdp_ep_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                 c_void_p, c_void_p, c_void_p]),
    "dwdp_ep_plan": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dwdp_ep_combine": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p]),
    "dwdp_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_void_p, c_void_p]),
    "dwdp_rope_append_kv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                    c_int, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dwdp_paged_attention_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "dwdp_paged_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                     c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dwdp_schedule": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p],
    ),
    "dwdp_packed_weight_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "dwdp_packed_scale_floats": (c_size_t, [c_int, c_int, c_int, c_int]),
    "dwdp_pack_weights": (
        c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]
    ),
    "dwdp_unpack_weights": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]
    ),
    "dwdp_moe_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int, c_int]),
    "dwdp_moe_experts": (
        c_int,
        [ctypes.POINTER(ExpertGroup), ctypes.POINTER(ExpertGroup), c_void_p, c_void_p, c_int64,
         c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
         c_void_p, c_void_p],
    ),
    "dwdp_moe_experts_indexed": (
        c_int,
        [ctypes.POINTER(ExpertGroup), ctypes.POINTER(ExpertGroup), c_void_p, c_void_p, c_int64,
         c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
         c_void_p, c_void_p],
    ),
    "dwdp_moe_shared_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "dwdp_moe_shared_expert": (
        c_int,
        [ctypes.POINTER(ExpertGroup), c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p,
         c_void_p],
    ),
    "dwdp_merge_gated": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_int, c_int, c_void_p, c_int, c_void_p]
    ),
    "dwdp_merge": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_int, c_void_p]
    ),
    "dwdp_moe_shared_parts": (c_int, [c_int64, c_int]),
    "dwdp_tensor_list_build": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, ctypes.POINTER(ExpertGroup),
         ctypes.POINTER(TensorListBases), ctypes.POINTER(TensorListHandle), c_void_p, c_void_p, c_void_p],
    ),
    "dwdp_grouped_moe": (
        c_int,
        [ctypes.POINTER(TensorListHandle), ctypes.POINTER(ExpertGroup), c_void_p, c_void_p, c_int64, c_int,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),

    # communication engine
    "dwdp_engine_last_error": (ctypes.c_char_p, []),
    "dwdp_ipc_handle_bytes": (c_size_t, []),
    "dwdp_export_ipc_handle": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_size_t)]),
    "dwdp_peer_can_access": (c_int, [c_int, c_int, ctypes.POINTER(c_int)]),
    "dwdp_engine_create": (c_int, [c_int, c_size_t, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "dwdp_engine_destroy": (c_int, [c_void_p]),
    "dwdp_engine_register_local": (c_int, [c_void_p, c_int, c_void_p, c_size_t]),
    "dwdp_engine_register_ipc": (c_int, [c_void_p, c_int, c_void_p, c_size_t, c_size_t, c_int]),
    "dwdp_engine_register_peer": (c_int, [c_void_p, c_int, c_void_p, c_size_t, c_int]),
    "dwdp_engine_prefetch": (c_int, [c_void_p, ctypes.POINTER(c_int), c_int, c_int, c_void_p]),
    "dwdp_engine_wait": (c_int, [c_void_p, c_int, c_void_p]),
    "dwdp_engine_prefetch_slices": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "dwdp_engine_resident_pointer": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "dwdp_engine_is_remote": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int)]),
    "dwdp_engine_release": (c_int, [c_void_p, c_int]),
    "dwdp_engine_synchronize": (c_int, [c_void_p]),
    "dwdp_engine_stats": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_ulonglong),
                                  ctypes.POINTER(ctypes.c_ulonglong), ctypes.POINTER(c_void_p)]),
    "dwdp_engine_set_copy_mode": (c_int, [c_void_p, c_int, c_int]),
    "dwdp_peer_copy_sm": (c_int, [c_void_p, c_int, c_void_p]),
    "dwdp_policy_decide": (c_int, [c_int, c_int, c_int, c_int, c_int]),
    "dwdp_sched_create": (c_int, [ctypes.POINTER(c_void_p)]),
    "dwdp_sched_destroy": (c_int, [c_void_p]),
    "dwdp_sched_submit": (c_int, [c_void_p, c_int, c_int]),
    "dwdp_sched_take": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int)]),
    "dwdp_sched_complete": (c_int, [c_void_p, c_int]),
    "dwdp_sched_fail": (c_int, [c_void_p, c_int, c_int]),
    "dwdp_sched_cancel": (c_int, [c_void_p, c_int]),
    "dwdp_sched_close": (c_int, [c_void_p]),
    "dwdp_sched_state": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
}

_lib = None
_lock = threading.Lock()


def load(path: pathlib.Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with argument types set."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = pathlib.Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"DWDP B200 extension not built: {p} is missing (run build.py); "
                "there is no CPU fallback"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    msg = load().dwdp_last_error()
    return msg.decode() if msg else ""


def engine_last_error() -> str:
    msg = load().dwdp_engine_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str, engine: bool = False) -> None:
    """Translate a C status code into the reference's exception types."""
    if rc == DWDP_OK:
        return
    msg = (engine_last_error() if engine else last_error()) or f"{what} failed with status {rc}"
    if rc == DWDP_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == DWDP_ERR_NOT_FOUND:
        raise KeyError(msg)
    if rc == DWDP_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == DWDP_ERR_DEVICE_TIMEOUT:
        raise TimeoutError(msg)
    if rc == DWDP_ERR_STATE:
        raise RuntimeError(msg)
    raise RuntimeError(msg)

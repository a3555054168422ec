"""CPU-side checks of the C ABI: the library loads without a GPU, exports every
entry point declared in include/*.h, the ctypes binding declares them all, and
host-side argument validation returns the documented status codes and messages
(no kernel is launched on these paths)."""
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared_in_headers() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(dwdp_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_in_headers()
    assert {"dwdp_router_topk", "dwdp_dispatch", "dwdp_moe_experts", "dwdp_merge"} <= names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    missing = [n for n in sorted(declared_in_headers()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_every_declared_symbol(pkg):
    assert declared_in_headers() <= set(pkg._lib.SIGNATURES)


def test_version_and_sizes(pkg):
    lib = pkg._lib.load()
    assert lib.dwdp_version() >= 100
    assert lib.dwdp_packed_weight_bytes(256, 128, 2, pkg._lib.DTYPE_FP8_E4M3) == 256 * 128 * 2
    assert lib.dwdp_packed_weight_bytes(256, 128, 1, pkg._lib.DTYPE_BF16) == 256 * 128 * 2
    assert lib.dwdp_packed_scale_floats(256, 128, 2, pkg._lib.SCALE_CHANNEL) == 512
    assert lib.dwdp_packed_scale_floats(256, 256, 1, pkg._lib.SCALE_BLOCK128) == 4
    assert lib.dwdp_dispatch_scratch_bytes(4096, 4, 60) >= 64 * 60 * 4
    assert lib.dwdp_moe_shared_parts(1, 5632) == 4
    assert lib.dwdp_moe_shared_parts(4096, 5632) == 1
    assert lib.dwdp_moe_shared_parts(1, 0) == 0
    assert lib.dwdp_moe_workspace_bytes(64, 4, 60, 1408, 5632) > 64 * 4 * 1408 * 2


def test_router_validation_errors(pkg):
    lib = pkg._lib.load()
    rc = lib.dwdp_router_topk(None, 2, None, 2, None, None, 4, 128, 300, 2, 1.0, 1, 1e-9,
                              None, None, None, None, None, None, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT
    assert "num_experts" in pkg._lib.last_error()
    rc = lib.dwdp_router_topk(None, 2, None, 2, None, None, 4, 128, 8, 9, 1.0, 1, 1e-9,
                              None, None, None, None, None, None, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT and "top_k" in pkg._lib.last_error()
    with pytest.raises(ValueError, match="top_k"):
        pkg._lib.check(rc, "router")


def test_dispatch_validation_errors(pkg):
    lib = pkg._lib.load()
    rc = lib.dwdp_dispatch(None, None, 4, 4, 2, 2000, None, None, None, None, None, None, None,
                           None, 0, None, None, None, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT and "num_experts" in pkg._lib.last_error()
    rc = lib.dwdp_dispatch(None, None, 4, 4, 2, 8, None, None, None, None, None, None, None,
                           None, 0, None, None, None, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT


def test_moe_and_merge_validation_errors(pkg):
    lib = pkg._lib.load()
    g = pkg._lib.ExpertGroup(num_experts=8, hidden_size=500, intermediate_size=256,
                             weight_dtype=pkg._lib.DTYPE_FP8_E4M3, scale_mode=pkg._lib.SCALE_CHANNEL)
    import ctypes
    rc = lib.dwdp_moe_experts(ctypes.byref(g), None, None, None, 4, 2, None, None, None, None,
                              None, None, None, 0, None, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT and "multiples of 128" in pkg._lib.last_error()
    g.hidden_size = 512
    rc = lib.dwdp_moe_experts(ctypes.byref(g), None, 1, 1, 4, 2, 1, 1, 1, None, 1, None, 1, 16, None, None)
    assert rc == pkg._lib.DWDP_ERR_CAPACITY and "workspace" in pkg._lib.last_error()
    rc = lib.dwdp_merge(None, None, None, 1, 4, 17, 128, None, pkg._lib.DTYPE_BF16, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT
    rc = lib.dwdp_pack_weights(None, 4, 100, 128, 1, 3, 1, None, None, None)
    assert rc == pkg._lib.DWDP_ERR_INVALID_ARGUMENT and "multiples of 128" in pkg._lib.last_error()


def test_tensor_list_validation_errors(pkg):
    import ctypes

    L = pkg._lib
    lib = L.load()
    g = L.ExpertGroup(num_experts=8, hidden_size=256, intermediate_size=256, weight_dtype=L.DTYPE_FP8_E4M3,
                      scale_mode=L.SCALE_CHANNEL)
    b = L.TensorListBases()
    h = L.TensorListHandle(capacity=2048, fields=1)
    rc = lib.dwdp_tensor_list_build(1, 1, 1, None, None, 8, ctypes.byref(g), ctypes.byref(b), ctypes.byref(h), 1,
                                    None, None)
    assert rc == L.DWDP_ERR_INVALID_ARGUMENT and "capacity" in L.last_error()
    h.capacity = 8
    rc = lib.dwdp_tensor_list_build(None, None, None, None, None, 8, ctypes.byref(g), ctypes.byref(b),
                                    ctypes.byref(h), 1, None, None)
    assert rc == L.DWDP_ERR_INVALID_ARGUMENT and "plan rows" in L.last_error()
    h.capacity = 0
    rc = lib.dwdp_grouped_moe(ctypes.byref(h), None, 1, 1, 4, 2, 1, None, 1, None, 1, 16, None, None)
    assert rc == L.DWDP_ERR_INVALID_ARGUMENT and "TensorList" in L.last_error()


def test_ops_refuse_cpu_tensors(pkg):
    import torch
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        pkg.ops.dispatch(torch.zeros(4, 2, dtype=torch.int64), torch.zeros(4, 2), 8)


def test_missing_library_fails_loudly(pkg, tmp_path):
    with pytest.raises(RuntimeError, match="not built"):
        pkg._lib.load(tmp_path / "nope.so")

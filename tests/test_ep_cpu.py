"""Host side of the expert-parallel decode path and the decode-step entry points, on
CPU: ownership ranges (the reference's owner map, DWDP/adapters/qwen15_moe.py:184-190),
buffer geometry, and the C ABI's argument validation (no kernel launches)."""
from __future__ import annotations

import pytest


@pytest.mark.parametrize("E,world", [(60, 1), (60, 2), (60, 8), (256, 8), (8, 8), (16, 3), (5, 8)])
def test_owned_ranges_partition_experts_like_the_reference(pkg, E, world):
    ep = pkg.ep
    seen = []
    for r in range(world):
        lo, hi = ep.ep_owned_range(r, E, world)
        assert all(ep.ep_owner(e, E, world) == r for e in range(lo, hi))
        seen += list(range(lo, hi))
    assert seen == list(range(E))
    # reference: target = clamp(e // ceil(E / world), max=world - 1)
    per = -(-E // world)
    assert [ep.ep_owner(e, E, world) for e in range(E)] == [min(e // per, world - 1) for e in range(E)]


def test_ep_owner_matches_dwdp_shard_owner(pkg):
    import importlib

    d = importlib.import_module("dwdp_b200.dwdp")
    for E, world in ((60, 2), (60, 8), (256, 8)):
        assert all(d.owner_of(e, E, world) == pkg.ep.ep_owner(e, E, world) for e in range(E))


def test_ep_buffer_geometry(pkg):
    lib = pkg._lib.load()
    a = lib.dwdp_ep_buffer_bytes(2, 2048, 256)
    b = lib.dwdp_ep_buffer_bytes(8, 2048, 256)
    assert 0 < a < b
    # receive rows for every source + return rows, bf16
    assert a >= 2 * 256 * 2048 * 2 + 256 * 2048 * 2
    off = lib.dwdp_ep_ret_offset(2, 2048, 256)
    assert off % 256 == 0 and off + 256 * 2048 * 2 <= a
    assert lib.dwdp_ep_buffer_bytes(9, 2048, 256) == 0 and lib.dwdp_ep_buffer_bytes(2, 0, 256) == 0


def test_ep_validation_errors(pkg):
    L = pkg._lib
    lib = L.load()
    # world out of range, rank out of range, too many slots
    assert lib.dwdp_ep_dispatch(None, None, None, 1, 4, 60, 0, 0, 2048, 256, None, None, None) == \
        L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_ep_dispatch(None, None, None, 1, 4, 60, 2, 2, 2048, 256, None, None, None) == \
        L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_ep_dispatch(None, None, None, 65, 4, 60, 2, 0, 2048, 256, None, None, None) == \
        L.DWDP_ERR_CAPACITY
    assert "capacity" in L.last_error()
    assert lib.dwdp_ep_plan(None, 2, 0, 2048, 256, 60, 0, 30, None, None, None, None, None, None, None, None,
                            None) == L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_ep_combine(None, 2, 0, 2048, 256, None, None, None, None, None, None) == \
        L.DWDP_ERR_INVALID_ARGUMENT


def test_decode_pieces_validation_errors(pkg):
    L = pkg._lib
    lib = L.load()
    assert lib.dwdp_add_rmsnorm(None, None, None, 1, 2047, 1e-6, None, None) == L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_rope_append_kv(None, None, None, None, 1, 8, 8, 16, 127, 16, 1e6, None, None, None, None,
                                   None) == L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_rope_append_kv(None, None, None, None, 1, 8, 0, 16, 128, 16, 1e6, None, None, None, None,
                                   None) == L.DWDP_ERR_INVALID_ARGUMENT  # no cache blocks
    assert lib.dwdp_paged_attention(None, None, None, None, None, 1, 8, 8, 16, 64, 16, 128, 1, 0.1, None, None,
                                    None, None) == L.DWDP_ERR_UNSUPPORTED
    assert lib.dwdp_paged_attention(None, None, None, None, None, 1, 8, 8, 16, 128, 16, 129, 1, 0.1, None, None,
                                    None, None) == L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_paged_attention(None, None, None, None, None, 1, 8, 0, 16, 128, 16, 128, 1, 0.1, None, None,
                                    None, None) == L.DWDP_ERR_INVALID_ARGUMENT
    assert lib.dwdp_paged_attention_workspace_bytes(4, 16, 8) >= 4 * 16 * 8 * 130 * 4


def test_paged_attention_split_choice(pkg):
    ops = pkg.ops
    for B in (1, 2, 8, 16, 64, 128, 256):
        s = ops.paged_attention_splits(B, 16, 2048, 16)
        assert 1 <= s <= 2048 // 16
    assert ops.paged_attention_splits(1, 16, 2048, 16) == 128  # 16-position chunks at B = 1
    # the fallback path (not 8/16/32 heads) sizes for ~4 CTAs per SM per (sequence, head)
    assert ops.paged_attention_splits(4, 4, 2048, 16) == 32


def test_kv_cache_manager_free_list(pkg):
    import torch

    m = pkg.decode.PagedKVCacheManager.__new__(pkg.decode.PagedKVCacheManager)
    # host bookkeeping only (no device storage): the reference's allocate/free contract
    import collections

    m.num_blocks, m.free_blocks, m.ref_counts = 4, collections.deque(range(4)), {}
    assert m.allocate(3) == [0, 1, 2]
    with pytest.raises(RuntimeError, match="Out of KV Cache memory"):
        m.allocate(2)
    m.free([1, 7])
    assert m.allocate(2) == [3, 1]
    assert set(m.used_blocks) == {0, 1, 2, 3}
    del torch

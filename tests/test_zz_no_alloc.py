"""The allocation-free dispatch entry point, ``dwdp_dispatch_noalloc``.

It exists for callers that cannot allocate device memory while they dispatch
(a serving loop held to a fixed memory budget, a plugin that only receives the
tensors of one call): its histogram scratch is a fixed array inside the library.
These checks call it through the C ABI and compare every output with the
ordinary ``dwdp_dispatch`` (caller-provided scratch) on two calls in a row, which
also shows that the contents left behind by the first call do not leak into the
second. The file name sorts last so a stop-at-first-failure run has already run
every other test."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _outputs(N, E, wdtype):
    mk = lambda n: torch.full((n,), -7, dtype=torch.int64, device=DEV)  # noqa: E731
    return {"counts": mk(E), "offsets": mk(E + 1), "perm": mk(N), "inv": mk(N), "ids": mk(N), "tok": mk(N),
            "w": torch.zeros(N, dtype=wdtype, device=DEV)}


def _call(lib, pkg, fn_name, ids, w, T, K, E, hidden, packed, out, scratch=None):
    args = [ids.data_ptr(), w.data_ptr(), pkg.ops.dtype_code(w.dtype), T, K, E,
            out["counts"].data_ptr(), out["offsets"].data_ptr(), out["perm"].data_ptr(), out["inv"].data_ptr(),
            out["ids"].data_ptr(), out["tok"].data_ptr(), out["w"].data_ptr(),
            hidden.data_ptr(), hidden.shape[1], packed.data_ptr()]
    if scratch is not None:
        args.append(scratch.data_ptr())
    args += [None, torch.cuda.current_stream().cuda_stream]
    rc = getattr(lib, fn_name)(*args)
    pkg._lib.check(rc, fn_name)


@pytest.mark.parametrize("T,E,K", [(4096, 60, 4), (513, 1024, 8)])
def test_noalloc_dispatch_matches_dispatch_twice(pkg, T, E, K):
    lib = pkg._lib.load()
    H = 256
    for call in range(2):  # two calls in a row, different routing each time
        g = torch.Generator().manual_seed(100 * call + T + E)
        ids = torch.randint(0, E, (T, K), generator=g).to(DEV)
        w = torch.rand(T, K, generator=g).to(DEV)
        hidden = torch.randn(T, H, generator=g).bfloat16().to(DEV)
        ref_out, got_out = _outputs(T * K, E, w.dtype), _outputs(T * K, E, w.dtype)
        ref_packed = torch.empty(T * K, H, dtype=torch.bfloat16, device=DEV)
        got_packed = torch.empty_like(ref_packed)
        scratch = torch.empty(pkg.ops.dispatch_scratch_bytes(T, K, E), dtype=torch.uint8, device=DEV)
        _call(lib, pkg, "dwdp_dispatch", ids, w, T, K, E, hidden, ref_packed, ref_out, scratch)
        _call(lib, pkg, "dwdp_dispatch_noalloc", ids, w, T, K, E, hidden, got_packed, got_out)
        torch.cuda.synchronize()
        for k in ref_out:
            assert torch.equal(ref_out[k], got_out[k]), f"call {call}: {k} differs"
        assert torch.equal(ref_packed, got_packed)
        # and both equal the reference's counting scatter
        ref = np.argsort(ids.reshape(-1).cpu().numpy(), kind="stable")
        assert np.array_equal(got_out["perm"].cpu().numpy(), ref)


def test_noalloc_dispatch_rejects_oversize(pkg):
    lib = pkg._lib.load()
    assert lib.dwdp_dispatch_noalloc_max_scratch_bytes() == 1 << 20
    T, K, E = 65537, 4, 1024  # ceil(T*K/256) * E * 4 bytes > 1 MiB
    rc = lib.dwdp_dispatch_noalloc(1, 1, pkg._lib.DTYPE_F32, T, K, E, 1, 1, 1, 1, 1, 1, 1, None, 0, None, None,
                                   None)
    assert rc == pkg._lib.DWDP_ERR_CAPACITY
    assert "exceed the fixed" in pkg._lib.last_error()

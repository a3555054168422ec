"""Expert-parallel decode path (token rows over NVLink peer memory) against the layer
with every expert local and against the CPU oracle. World 1 runs the same kernels on one
GPU; world 2 needs two GPUs. Every result must be bit-identical to the local layer (run
with its shared expert in separate launches, as the EP path runs it): a row's expert
arithmetic does not depend on which rows share its tile, and the merge adds the k slots
in the same order. Ranks may run different token counts, none included."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, H, I, K, Is = 16, 512, 256, 4, 512


def _weights(seed=11):
    g = torch.Generator().manual_seed(seed)
    wr = (torch.randn(E, H, generator=g) / H**0.5).bfloat16()
    mats = [(torch.randn(I, H, generator=g) * 0.02, torch.randn(I, H, generator=g) * 0.02,
             torch.randn(H, I, generator=g) * 0.02) for _ in range(E)]
    shared = (torch.randn(Is, H, generator=g) * 0.02, torch.randn(Is, H, generator=g) * 0.02,
              torch.randn(H, Is, generator=g) * 0.02)
    gate = (torch.randn(H, generator=g) * 0.02).bfloat16()
    return wr, mats, shared, gate


def _layers(pkg, ep, rank, world, dev, exchange):
    wr, mats, shared, gate = _weights()
    full = pkg.ExpertWeightStore(E, H, I, device=dev)
    for e in range(E):
        full.load_expert(e, *mats[e])
    lo, hi = ep.ep_owned_range(rank, E, world)
    local = pkg.ExpertWeightStore(max(1, hi - lo), H, I, device=dev)
    for e in range(lo, hi):
        local.load_expert(e - lo, *mats[e])
    sh = pkg.ExpertWeightStore(1, H, Is, device=dev)
    sh.load_expert(0, *shared)
    wr, gate = wr.to(dev), gate.to(dev)
    ref = pkg.MoELayer(wr, full, K, shared_expert=sh, shared_gate_weight=gate)
    epl = ep.ExpertParallelMoE(wr, local, K, exchange, shared_expert=sh, shared_gate_weight=gate)
    return ref, epl


# per-step token counts of rank r: equal, then unequal, then one rank with none
STEPS = [(1, 1), (5, 5), (64, 64), (5, 3), (0, 7), (1, 0)]


def _check(pkg, ep, rank, world, dev, exchange):
    ref, epl = _layers(pkg, ep, rank, world, dev, exchange)
    results = []
    for it, Ts in enumerate(STEPS):
        T = Ts[rank % 2]
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(100 * rank + it)).bfloat16().to(dev)
        y_ref = ref(x) if T else torch.empty(0, H, dtype=torch.bfloat16, device=dev)
        y = epl(x)
        torch.cuda.synchronize()
        results.append((T, bool(torch.equal(y, y_ref)), epl.read_status(T)[0]))
    # graph capture of two chained EP layers, replayed twice
    T = 8
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(7 + rank)).bfloat16().to(dev)
    ws = epl.workspace(T)
    y1, y2 = torch.empty_like(x), torch.empty_like(x)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        epl.run(x, ws, y1)
        epl.run(y1, ws, y2)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = y2.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        epl.run(x, ws, y1)
        epl.run(y1, ws, y2)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    results.append(("graph", bool(torch.equal(y2, eager)), epl.read_status(T)[0]))
    return results


def test_ep_world1_matches_local_layer(pkg):
    ep = pkg.ep
    dev = torch.device("cuda", 0)
    ex = ep.EPExchange(1, 0, H, 64, K, dev)
    for T, ok, st in _check(pkg, ep, 0, 1, dev, ex):
        assert st == 0, f"T={T}: status {st}"
        assert ok, f"T={T}: EP output differs from the local layer"


def test_ep_world1_matches_oracle(pkg, orc):
    """The EP layer against the CPU oracle of the reference's EP forward
    (DWDP/adapters/qwen15_moe.py:164-243: the same routed experts and shared expert)."""
    ep = pkg.ep
    dev = torch.device("cuda", 0)
    ex = ep.EPExchange(1, 0, H, 64, K, dev)
    ref, epl = _layers(pkg, ep, 0, 1, dev, ex)
    for T in (1, 13, 64):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).bfloat16()
        y = epl(x.to(dev))
        torch.cuda.synchronize()
        assert epl.read_status(T)[0] == 0
        r = epl.workspace(T)["router"]
        experts = [tuple(t.cpu() for t in ref.experts.dequantized(e)) for e in range(E)]
        shared = tuple(t.cpu() for t in ref.shared_expert.dequantized(0))
        want = orc.moe_forward(x.float(), r.topk_indices.cpu(), r.topk_weights.cpu(), experts, shared=shared,
                               shared_gate=r.shared_gate.cpu())
        assert orc.rel_frobenius(y.float().cpu(), want) < 2e-2


def test_ep_plan_wait_runs_out(pkg):
    """A world-2 exchange on one GPU whose second rank never sends: the owner's bounded wait
    gives up (about a second), records DWDP_ERR_DEVICE_TIMEOUT in the status word and the
    kernel returns; the context stays usable. Nothing here writes to a peer."""
    import ctypes

    ep = pkg.ep
    dev = torch.device("cuda", 0)
    ex = ep.EPExchange(2, 0, H, 8, K, dev)
    El = E // 2
    counts = torch.zeros(El, dtype=torch.int64, device=dev)
    offsets = torch.zeros(El + 1, dtype=torch.int64, device=dev)
    cap_rows = 2 * ex.capacity
    src = torch.zeros(cap_rows, dtype=torch.int32, device=dev)
    w = torch.zeros(cap_rows, dtype=torch.float32, device=dev)
    ret = torch.zeros(cap_rows, dtype=torch.int32, device=dev)
    total = torch.zeros(1, dtype=torch.int32, device=dev)
    packed = torch.zeros(cap_rows, H, dtype=torch.bfloat16, device=dev)
    st = torch.zeros(4, dtype=torch.int32, device=dev)
    lib = pkg._lib.load()
    rc = lib.dwdp_ep_plan(ex.buffer.data_ptr(), 2, 0, H, ex.capacity, E, 0, El, counts.data_ptr(),
                          offsets.data_ptr(), src.data_ptr(), w.data_ptr(), ret.data_ptr(), total.data_ptr(),
                          packed.data_ptr(), st.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    pkg._lib.check(rc, "ep_plan")
    torch.cuda.synchronize()
    assert st.cpu().tolist()[0] == pkg._lib.DWDP_ERR_DEVICE_TIMEOUT
    assert int(total.item()) == 0
    assert torch.ones(4, device=dev).sum().item() == 4.0  # the context still runs work


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        ex = pkg.ep.EPExchange(world, rank, H, 64, K, dev)
        ex.connect()
        res = _check(pkg, pkg.ep, rank, world, dev, ex)
        dist.barrier()
        ex.close()
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_world2_matches_local_layer():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in out:
        assert not isinstance(res, str), f"rank {rank}: {res}"
        for T, ok, st in res:
            assert st == 0, f"rank {rank} T={T}: status {st}"
            assert ok, f"rank {rank} T={T}: EP output differs from the local layer"

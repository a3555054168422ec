"""Expert-parallel decode path (token rows over NVLink peer memory) against the layer
with every expert local. World 1 runs the same kernels on one GPU; world 2 needs two
GPUs (gpurun --gpus 2). Every result must be bit-identical to the local layer: a row's
expert arithmetic does not depend on which rows share its tile, and the merge adds the
k slots in the same order."""
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


def _check(pkg, ep, rank, world, dev, exchange):
    ref, epl = _layers(pkg, ep, rank, world, dev, exchange)
    results = []
    for it, T in enumerate((1, 5, 64, 5, 1)):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(100 * rank + it)).bfloat16().to(dev)
        y_ref = ref(x)
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

"""DWDP on 2+ GPUs: experts sharded across ranks, remote experts prefetched over
NVLink (CUDA IPC + copy engine) into staging, then the same grouped GEMM. Each
rank's output must be bit-identical to the layer run with every expert local.
Runs only where at least two GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

need2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, block_scales=False):
    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    import importlib
    d = importlib.import_module("dwdp_b200.dwdp")
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        E, H, I, K, Is = 16, 512, 256, 4, 512
        g = torch.Generator().manual_seed(11)
        wr = (torch.randn(E, H, generator=g) / H**0.5).bfloat16().to(dev)
        gates = [torch.randn(I, H, generator=g) * 0.02 for _ in range(E)]
        ups = [torch.randn(I, H, generator=g) * 0.02 for _ in range(E)]
        downs = [torch.randn(H, I, generator=g) * 0.02 for _ in range(E)]
        mode = pkg._lib.SCALE_BLOCK128 if block_scales else pkg._lib.SCALE_CHANNEL
        full = pkg.ExpertWeightStore(E, H, I, device=dev, scale_mode=mode)
        shard = d.ShardedExpertStore(E, H, I, rank=rank, world_size=world, device=dev, num_buffers=2,
                                     scale_mode=mode)
        for e in range(E):
            full.load_expert(e, gates[e], ups[e], downs[e])
            shard.load_expert(e, gates[e], ups[e], downs[e])
        shard.connect()
        x = torch.randn(200, H, generator=torch.Generator().manual_seed(100 + rank)).bfloat16().to(dev)
        ref = pkg.MoELayer(wr, full, K)(x)
        outs = []
        for i, buf in enumerate((0, 1, 0)):
            shard.engine.set_copy_mode("sm" if i == 1 else "engine", 64)  # both copy mechanisms
            shard.prefetch(buf)
            shard.wait(buf)
            shard.select_buffer(buf)
            layer = pkg.MoELayer(wr, shard, K)
            outs.append(layer(x))
        torch.cuda.synchronize()
        ok = all(torch.equal(o, ref) for o in outs)
        st = shard.engine.stats()
        q.put((rank, ok, st["bytes_copied"], len(shard.remote) * shard.slab_bytes))
        dist.barrier()
        shard.shutdown()
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc), 0, 0))


@need2
@pytest.mark.parametrize("block_scales", [False, True], ids=["channel_scales", "block128_scales"])
def test_dwdp_sharded_layer_matches_local(block_scales):
    """Per-channel weights (the Qwen shape's) and 128x128 block-scaled weights (the Mixtral /
    DeepSeek shapes'): staged copies carry the slab's scales with its tiles."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, block_scales)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, copied, remote in res:
        assert ok is True, f"rank {rank}: {ok}"
        assert copied == 3 * remote  # three prefetches of every remote expert


def test_engine_reference_surface_single_gpu(pkg):
    """The reference's engine calls on one GPU (a same-device "peer" stands in for a remote
    owner): prefetch(id) stages into the next buffer, which is not resident until
    swap_buffers(); then get_weight(id) is a staged copy holding the owner's bytes."""
    import ctypes

    dev = torch.device("cuda", 0)
    nbytes = 3 << 20
    local = torch.arange(nbytes, dtype=torch.int64, device=dev).to(torch.uint8)
    remote = (torch.arange(nbytes, dtype=torch.int64, device=dev) * 7 + 3).to(torch.uint8)
    eng = pkg.communication.CommunicationEngine(0)
    eng.initialize(4 << 20)
    eng.register_expert(0, local.data_ptr(), nbytes)
    eng.register_peer_expert(1, remote.data_ptr(), nbytes, 0)
    assert eng.get_weight(0) == local.data_ptr()
    assert not eng.is_resident(1)
    eng.prefetch(1)
    assert not eng.is_resident(1)
    with pytest.raises(RuntimeError):
        eng.get_resident_pointer(1)  # staged in the next buffer only
    eng.swap_buffers()
    assert eng.is_resident(1)
    ptr = eng.get_weight(1)
    assert ptr not in (0, remote.data_ptr())
    torch.cuda.synchronize()
    host = torch.empty(nbytes, dtype=torch.uint8)
    cudart = ctypes.CDLL("libcudart.so.12")
    assert cudart.cudaMemcpy(ctypes.c_void_p(host.data_ptr()), ctypes.c_void_p(ptr), ctypes.c_size_t(nbytes), 2) == 0
    assert torch.equal(host, remote.cpu())
    eng.swap_buffers()
    assert not eng.is_resident(1)
    eng.shutdown()


def test_engine_sm_copy_mode_single_gpu(pkg):
    """DWDP_COPY_SM: the prefetch copies run as one SM kernel; every byte staged, ragged sizes
    (not a multiple of 16 bytes) included, for several experts and CTA counts."""
    import ctypes

    dev = torch.device("cuda", 0)
    sizes = [(1 << 20) + 5, 3 << 20, 4096 + 16, 7]
    srcs = [((torch.arange(n, dtype=torch.int64, device=dev) * (3 + i) + i) % 251).to(torch.uint8)
            for i, n in enumerate(sizes)]
    cudart = ctypes.CDLL("libcudart.so.12")
    for ctas in (1, 148):
        eng = pkg.communication.CommunicationEngine(0)
        eng.initialize(4 << 20)
        for i, (n, t) in enumerate(zip(sizes, srcs)):
            eng.register_peer_expert(i, t.data_ptr(), n, 0)
        eng.set_copy_mode("sm", ctas)
        for i in range(len(sizes)):
            eng.prefetch(i)
        eng.swap_buffers()
        torch.cuda.synchronize()
        for i, (n, t) in enumerate(zip(sizes, srcs)):
            host = torch.empty(n, dtype=torch.uint8)
            assert cudart.cudaMemcpy(ctypes.c_void_p(host.data_ptr()), ctypes.c_void_p(eng.get_weight(i)),
                                     ctypes.c_size_t(n), 2) == 0
            assert torch.equal(host, t.cpu()), (ctas, i)
        with pytest.raises(ValueError):
            eng.set_copy_mode("dma")
        eng.shutdown()


@pytest.mark.parametrize("mode", ["engine", "sm"])
def test_engine_executes_the_planners_slices_single_gpu(pkg, mode):
    """The DWDP planner's plan (2 MiB slices, rotated start slice, priorities) executed by the
    engine in the TransferScheduler's order stages every remote expert's bytes exactly; the
    remote owners are same-device buffers standing in for peers."""
    st = pkg.stages
    dev = torch.device("cuda", 0)
    E, G, rank = 12, 4, 1
    sizes = [(5 << 20) + 4096 * e for e in range(E)]  # ragged: three slices, the last one short
    srcs = [((torch.arange(n, dtype=torch.int64, device=dev) * (e + 3) + e) % 251).to(torch.uint8)
            for e, n in enumerate(sizes)]
    planner = st.DWDPCommunicationPlanner(st.CommunicationPlannerConfig("dwdp", G, rank),
                                          bytes_per_expert=lambda e: sizes[e], peer_access=lambda s, d: True)
    plan = planner(type("EP", (), {"expert_queue": torch.zeros(E, dtype=torch.int64, device=dev)})())
    assert {d.count for d in plan.communication_descriptors} >= {2 << 20}
    eng = pkg.communication.CommunicationEngine(0)
    eng.initialize(max(sizes), len(plan.remote_expert_ids), 2)
    owners = {e: min(e // -(-E // G), G - 1) for e in range(E)}
    for e in range(E):
        if owners[e] == rank:
            eng.register_expert(e, srcs[e].data_ptr(), sizes[e])
        else:
            eng.register_peer_expert(e, srcs[e].data_ptr(), sizes[e], 0)
    if mode == "sm":
        eng.set_copy_mode("sm", 16)
    import ctypes

    order = eng.execute_plan(plan, buffer=1)
    prios = [d.priority for d in order]
    assert prios == sorted(prios, reverse=True)  # highest priority first
    eng.wait_buffer(1)
    torch.cuda.synchronize()
    for e in plan.remote_expert_ids.tolist():
        ptr = eng.get_resident_pointer(e, buffer=1)
        got = torch.empty(sizes[e], dtype=torch.uint8, device=dev)
        cudart = ctypes.CDLL("libcudart.so.12")
        assert cudart.cudaMemcpy(ctypes.c_void_p(got.data_ptr()), ctypes.c_void_p(ptr), ctypes.c_size_t(sizes[e]),
                                 3) == 0
        assert torch.equal(got, srcs[e]), f"expert {e}"
    eng.shutdown()

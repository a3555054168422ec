"""Host-side DWDP logic on CPU: expert ownership, the shard-record exchange over
a 2-rank gloo group, the transfer scheduler and the path policy (no GPU)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_ownership_partitions_experts(pkg):
    import importlib
    d = importlib.import_module("dwdp_b200.dwdp")
    for E, G in [(60, 8), (8, 2), (256, 8), (7, 4), (60, 1)]:
        seen = sorted(e for r in range(G) for e in d.owned_experts(r, E, G))
        assert seen == list(range(E))
        # contiguous blocks of ceil(E/G), as DWDP/comms_planner/expert_parallel.py:120-122
        for e in range(E):
            assert d.owner_of(e, E, G) == e // -(-E // G)


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    import importlib
    d = importlib.import_module("dwdp_b200.dwdp")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rec = d.ShardRecord(rank, rank, d.owned_experts(rank, 10, world), 4096, bytes([rank]) * 72)
    out = d.exchange_shard_records(rec)
    q.put((rank, [(r.rank, r.owned, r.ipc_blob[:1]) for r in out]))
    dist.destroy_process_group()


def test_shard_record_exchange_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    assert [r[0] for r in res[0]] == [0, 1]
    assert res[0][0][1] == [0, 1, 2, 3, 4] and res[0][1][1] == [5, 6, 7, 8, 9]
    assert res[0][1][2] == bytes([1])


def _silent_worker(rank, world, port, q):
    """Rank 1 never joins the exchange: rank 0 must fail with a timeout, not hang."""
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 0:
        import __graft_entry__
        __graft_entry__.load_package()
        import importlib
        d = importlib.import_module("dwdp_b200.dwdp")
        try:
            d.exchange_shard_records(d.ShardRecord(0, 0, [0], 16, b"x"))
            q.put("returned")
        except Exception as exc:  # noqa: BLE001 - the failure is the point
            q.put(type(exc).__name__)
    else:
        import time
        time.sleep(15)
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def test_exchange_fails_when_a_rank_never_joins():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_silent_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert outcome != "returned"


def test_transfer_scheduler_contract(pkg):
    import importlib
    c = importlib.import_module("dwdp_b200.communication")
    s = c.TransferScheduler()
    s.submit(3, priority=1)
    s.submit(5, priority=9)
    s.submit(3, priority=7)  # coalesced with the queued transfer of expert 3
    s.submit(6, priority=9)  # same priority as 5: FIFO
    assert [s.take(10), s.take(10), s.take(10)] == [5, 6, 3]
    s.fail(3, retryable=True)
    assert s.state(3) == (c.TransferState.QUEUED, 1)
    assert s.take(10) == 3
    s.fail(3, retryable=True)
    assert s.take(10) == 3
    s.fail(3, retryable=True)  # third failure: retries exhausted
    assert s.state(3)[0] == c.TransferState.FAILED
    s.complete(5)
    assert s.state(5)[0] == c.TransferState.COMPLETED
    with pytest.raises(RuntimeError):
        s.complete(5)  # illegal transition
    s.submit(8, 0)
    s.cancel(8)
    assert s.state(8)[0] == c.TransferState.CANCELLED
    with pytest.raises(TimeoutError):
        s.take(20)  # nothing queued: bounded wait
    s.complete(6)
    with pytest.raises(ValueError):
        s.submit(-1)
    s.close()
    assert s.take(10) is None
    with pytest.raises(RuntimeError):
        s.submit(1)


def test_policy_table(pkg):
    import importlib
    c = importlib.import_module("dwdp_b200.communication")
    p = c.CommunicationPolicy(local_gpu=0)
    assert p.decide(owner_gpu=3, resident=c.ResidentState.STAGED) == c.CommunicationPath.LOCAL
    assert p.decide(owner_gpu=3, has_ipc_handle=True, peer_access=True) == c.CommunicationPath.IPC
    assert p.decide(owner_gpu=3, peer_access=True) == c.CommunicationPath.P2P
    assert p.decide(owner_gpu=3, peer_access=False) == c.CommunicationPath.COPY
    assert p.decide(owner_gpu=0) == c.CommunicationPath.COPY


def test_engine_reference_surface_bookkeeping(pkg):
    """The reference's CommunicationEngine surface before any device work: initialize(staging_bytes)
    defers the staging allocation until the experts are known; local experts are resident and
    need neither a copy nor a wait; an oversized remote expert is refused."""
    eng = pkg.communication.CommunicationEngine(0)
    assert not eng.initialized()
    eng.initialize(1 << 20)
    assert eng.initialized()
    eng.register_expert(3, 0x1000, 4096)
    assert eng.is_resident(3)
    eng.prefetch(3)  # local: nothing to copy
    eng.wait(3)
    assert eng.current_buffer == 0 and eng.next_buffer == 1
    with pytest.raises(ValueError):
        eng.register_peer_expert(4, 0x2000, 2 << 20, 1)
    with pytest.raises(RuntimeError):
        eng.wait(5)  # never prefetched


def test_engine_issue_order_follows_the_scheduler(pkg):
    """The engine issues a plan's slices expert by expert in the TransferScheduler's order
    (priority, highest first), each expert's slices in the planner's rotated order."""
    st = pkg.stages
    E, G, rank = 16, 4, 2
    sizes = [(3 << 20) + e for e in range(E)]
    plan = st.DWDPCommunicationPlanner(st.CommunicationPlannerConfig("dwdp", G, rank),
                                       bytes_per_expert=lambda e: sizes[e], peer_access=lambda s, d: True)(
        type("EP", (), {"expert_queue": torch.zeros(E, dtype=torch.int64)})())
    order = pkg.communication.CommunicationEngine(0).issue_order(plan)
    assert sorted(d.descriptor_id for d in order) == list(range(len(plan.communication_descriptors)))
    experts = []
    for d in order:
        if not experts or experts[-1] != d.source_expert_id:
            experts.append(d.source_expert_id)
    assert experts == plan.remote_expert_ids.tolist()  # priority E - position: ascending remote ids
    first = [d for d in order if d.source_expert_id == experts[0]]
    assert first[0].start == (rank % len(first)) * (2 << 20)  # rotated start slice
    assert sum(d.count for d in first) == sizes[experts[0]]

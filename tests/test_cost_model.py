"""Communication cost model (the reference's CommunicationCostModel filled from a measured
link instead of constants) and the sharded planner that attaches it, on CPU."""
from __future__ import annotations

import dataclasses

import pytest
import torch


def test_dataclass_fields_match_the_reference(pkg):
    cm = pkg.cost_model
    # DWDP/comms_planner/cost_model.py:6-29
    assert [f.name for f in dataclasses.fields(cm.CommunicationCostEstimate)] == [
        "descriptor_id", "estimated_bytes", "estimated_latency_us", "estimated_bandwidth_gbps",
        "communication_priority", "critical_path_us", "transfer_duration_us", "prefetch_window_us",
        "overlap_estimate_us"]
    assert [f.name for f in dataclasses.fields(cm.CommunicationCostModel)] == [
        "estimates", "total_estimated_bytes", "total_estimated_latency_us", "critical_path_us",
        "estimated_bandwidth_gbps"]


def test_fit_link_recovers_latency_and_bandwidth(pkg):
    cm = pkg.cost_model
    lat, bw = 7.5, 480.0  # us, GB/s
    samples = [(n, lat + n / (bw * 1e3)) for n in (1 << 20, 8 << 20, 64 << 20)]
    link = cm.fit_link(samples, streams=1)
    assert link.latency_us == pytest.approx(lat, rel=1e-6)
    assert link.bandwidth_gbps == pytest.approx(bw, rel=1e-6)
    with pytest.raises(ValueError):
        cm.fit_link([(1 << 20, 5.0)])
    with pytest.raises(ValueError):
        cm.fit_link([(1 << 20, 5.0), (1 << 20, 6.0)])


def test_batch_time_is_stream_or_link_bound(pkg):
    cm = pkg.cost_model
    link = cm.LinkProfile(latency_us=10.0, bandwidth_gbps=150.0, aggregate_gbps=480.0, streams=4)
    n = 8_650_000
    assert link.batch_us([n]) == pytest.approx(link.copy_us(n))          # one copy: its stream
    many = [n] * 30
    assert link.batch_us(many) == pytest.approx(max(8 * link.copy_us(n), 10.0 + 30 * n / 480e3))
    assert link.batch_us([]) == 0.0


def test_cost_model_window_and_critical_path(pkg):
    cm = pkg.cost_model
    link = cm.LinkProfile(latency_us=10.0, bandwidth_gbps=150.0, aggregate_gbps=480.0, streams=4)
    n = 8_650_000
    ids = list(range(30))
    total = link.batch_us([n] * 30)
    hidden = cm.build_cost_model(ids, n, link, prefetch_window_us=total + 100.0)
    assert hidden.critical_path_us == 0.0 and hidden.total_estimated_bytes == 30 * n
    assert len(hidden.estimates) == 30 and hidden.estimates[0].overlap_estimate_us == pytest.approx(total)
    exposed = cm.build_cost_model(ids, n, link, prefetch_window_us=200.0)
    assert exposed.critical_path_us == pytest.approx(total - 200.0)
    assert exposed.estimates[3].transfer_duration_us == pytest.approx(link.copy_us(n))
    assert exposed.estimated_bandwidth_gbps == 480.0


def test_decode_path_choice(pkg):
    cm = pkg.cost_model
    link = cm.LinkProfile(latency_us=10.0, bandwidth_gbps=150.0, aggregate_gbps=480.0, streams=4)
    kw = dict(top_k=4, hidden_size=2048, world_size=2, remote_experts=30, bytes_per_expert=8_650_000,
              link=link, ep_exchange_us=20.0)
    small = cm.choose_decode_path(1, local_layer_us=55.0, **kw)
    assert small.path == "ep" and small.ep_us < small.dwdp_us
    # prefill: the previous layer's 700 us hide the prefetch; EP would move 16 k rows twice
    big = cm.choose_decode_path(4096, local_layer_us=700.0, prefetch_window_us=700.0, **kw)
    assert big.path == "dwdp"
    single = cm.choose_decode_path(8, local_layer_us=80.0, **{**kw, "world_size": 1, "remote_experts": 0})
    assert single.ep_us == single.dwdp_us == 80.0


def test_dwdp_planner_partitions_and_attaches_the_model(pkg):
    st, cm = pkg.stages, pkg.cost_model
    link = cm.LinkProfile(latency_us=10.0, bandwidth_gbps=150.0, aggregate_gbps=480.0, streams=4)
    plan = torch.zeros(60, dtype=torch.int64)
    ex = type("EP", (), {"expert_queue": plan})()
    for rank in range(2):
        planner = st.DWDPCommunicationPlanner(st.CommunicationPlannerConfig("dwdp", 2, rank), link=link,
                                              bytes_per_expert=8_650_000, prefetch_window_us=500.0)
        cp = planner(ex)
        assert cp.local_expert_ids.tolist() == list(range(30 * rank, 30 * rank + 30))
        assert sorted(cp.remote_expert_ids.tolist() + cp.local_expert_ids.tolist()) == list(range(60))
        assert cp.cost_model.total_estimated_bytes == 30 * 8_650_000
    assert st._lookup("planner", "dwdp") is st.DWDPCommunicationPlanner
    static = st.StaticCommunicationPlanner()(ex)
    assert static.remote_expert_ids.numel() == 0 and static.cost_model.estimates == ()

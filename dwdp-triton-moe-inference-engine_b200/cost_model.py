"""Communication cost model for the DWDP prefetch (and the EP alternative at decode sizes).

The reference carries a ``CommunicationCostModel`` on every communication plan
(``DWDP/comms_planner/cost_model.py:6-29``), but fills it with constants: each estimate
gets ``default_link_latency_us`` / ``default_link_bandwidth_gbps`` (both 0 by default,
``DWDP/comms_planner/config.py:35-36``) and zero durations, windows and critical path
(``DWDP/comms_planner/expert_parallel.py:248-260, 298-304``). Here the same dataclasses
(same field names) are filled from a measured link:

* ``LinkProfile``: latency + bytes / bandwidth of one peer copy, fitted from timed copies of
  two sizes (``measure_link``) or given;
* ``build_cost_model``: one estimate per remote expert, copies spread over the engine's
  copy streams (the engine issues one copy per expert, round-robin over its streams), the
  previous layer's compute time as the prefetch window, and the exposed (critical-path)
  transfer time = max(0, transfer - window);
* ``choose_decode_path``: DWDP (move every remote expert's weights) against EP (move the
  tokens' rows to the owners and back) for a batch size, from the same link profile and
  the per-layer times the caller measured or estimated; the reference switches on a fixed
  ``ep_batch_size_threshold`` (``DWDP/runtime/config.py:31``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(slots=True)
class CommunicationCostEstimate:
    """Cost of one transfer descriptor (field names of the reference's estimate)."""

    descriptor_id: int
    estimated_bytes: int
    estimated_latency_us: float
    estimated_bandwidth_gbps: float
    communication_priority: int
    critical_path_us: float
    transfer_duration_us: float
    prefetch_window_us: float
    overlap_estimate_us: float


@dataclass(slots=True)
class CommunicationCostModel:
    """Aggregate over a plan's transfers (field names of the reference's model)."""

    estimates: tuple[CommunicationCostEstimate, ...]
    total_estimated_bytes: int
    total_estimated_latency_us: float
    critical_path_us: float
    estimated_bandwidth_gbps: float


@dataclass(frozen=True, slots=True)
class LinkProfile:
    """One peer-to-peer copy of n bytes takes latency_us + n / (bandwidth_gbps * 1e3) us
    (GB/s = 1e9 bytes/s). ``streams`` copies run side by side (the engine's copy streams),
    sharing ``aggregate_gbps`` (the link rate all of them together reach)."""

    latency_us: float
    bandwidth_gbps: float
    aggregate_gbps: float
    streams: int = 4

    def copy_us(self, nbytes: int) -> float:
        return self.latency_us + nbytes / (self.bandwidth_gbps * 1e3) if nbytes > 0 else 0.0

    def batch_us(self, sizes: list[int]) -> float:
        """Time for a batch of copies issued round-robin over the streams: the slower of the
        longest stream's serial chain and the aggregate link limit."""
        if not sizes:
            return 0.0
        chains = [0.0] * max(1, self.streams)
        for i, n in enumerate(sizes):
            chains[i % len(chains)] += self.copy_us(n)
        link = self.latency_us + sum(sizes) / (self.aggregate_gbps * 1e3)
        return max(max(chains), link)


def fit_link(samples: list[tuple[int, float]], *, streams: int = 4,
             aggregate_gbps: float | None = None) -> LinkProfile:
    """Least-squares latency + bytes/bandwidth from (bytes, microseconds) single-copy samples."""
    if len(samples) < 2:
        raise ValueError("need copies of at least two sizes")
    n = len(samples)
    mx = sum(b for b, _ in samples) / n
    my = sum(t for _, t in samples) / n
    sxx = sum((b - mx) ** 2 for b, _ in samples)
    if sxx <= 0:
        raise ValueError("need copies of at least two different sizes")
    slope = sum((b - mx) * (t - my) for b, t in samples) / sxx  # us per byte
    if slope <= 0:
        raise ValueError("copy time does not grow with size")
    latency = max(0.0, my - slope * mx)
    bw = 1.0 / (slope * 1e3)  # GB/s
    return LinkProfile(latency_us=latency, bandwidth_gbps=bw, aggregate_gbps=aggregate_gbps or bw * streams,
                       streams=streams)


def build_cost_model(remote_expert_ids: list[int], bytes_per_expert: int, link: LinkProfile, *,
                     prefetch_window_us: float = 0.0, priorities: list[int] | None = None
                     ) -> CommunicationCostModel:
    """Estimates for prefetching ``remote_expert_ids`` (one copy each) while the previous
    layer computes for ``prefetch_window_us``. critical_path_us is the part of the batch
    that the window does not hide."""
    sizes = [bytes_per_expert] * len(remote_expert_ids)
    total_us = link.batch_us(sizes)
    overlap = min(total_us, max(0.0, prefetch_window_us))
    exposed = total_us - overlap
    per = link.copy_us(bytes_per_expert)
    pr = priorities if priorities is not None else [0] * len(remote_expert_ids)
    est = tuple(
        CommunicationCostEstimate(
            descriptor_id=i, estimated_bytes=bytes_per_expert, estimated_latency_us=link.latency_us,
            estimated_bandwidth_gbps=link.bandwidth_gbps, communication_priority=pr[i],
            critical_path_us=exposed, transfer_duration_us=per, prefetch_window_us=prefetch_window_us,
            overlap_estimate_us=overlap)
        for i, _ in enumerate(remote_expert_ids))
    return CommunicationCostModel(estimates=est, total_estimated_bytes=sum(sizes), total_estimated_latency_us=total_us,
                                  critical_path_us=exposed, estimated_bandwidth_gbps=link.aggregate_gbps)


def build_descriptor_cost_model(descriptors, link: LinkProfile, *, prefetch_window_us: float = 0.0
                                ) -> CommunicationCostModel:
    """One estimate per communication descriptor (a slice or a whole expert) of a plan, the
    copies issued in descriptor order round-robin over the engine's copy streams."""
    sizes = [int(d.count) for d in descriptors]
    total_us = link.batch_us(sizes)
    overlap = min(total_us, max(0.0, prefetch_window_us))
    exposed = total_us - overlap
    est = tuple(
        CommunicationCostEstimate(
            descriptor_id=d.descriptor_id, estimated_bytes=int(d.count), estimated_latency_us=link.latency_us,
            estimated_bandwidth_gbps=link.bandwidth_gbps, communication_priority=d.priority,
            critical_path_us=exposed, transfer_duration_us=link.copy_us(int(d.count)),
            prefetch_window_us=prefetch_window_us, overlap_estimate_us=overlap)
        for d in descriptors)
    return CommunicationCostModel(estimates=est, total_estimated_bytes=sum(sizes), total_estimated_latency_us=total_us,
                                  critical_path_us=exposed, estimated_bandwidth_gbps=link.aggregate_gbps)


@dataclass(frozen=True, slots=True)
class DecodePathChoice:
    path: str  # "ep" | "dwdp"
    ep_us: float
    dwdp_us: float


def choose_decode_path(num_tokens: int, top_k: int, hidden_size: int, world_size: int, *,
                       remote_experts: int, bytes_per_expert: int, link: LinkProfile,
                       local_layer_us: float, ep_exchange_us: float, prefetch_window_us: float = 0.0
                       ) -> DecodePathChoice:
    """Per-layer time of the two multi-GPU decode paths for ``num_tokens`` tokens per rank:
    DWDP = the local layer + the prefetch the window does not hide; EP = the local layer +
    the exchange's fixed cost (``ep_exchange_us``: its extra launches and waits, measured) +
    the rows' transfer both ways (bf16, (G-1)/G of them remote)."""
    dwdp = local_layer_us + build_cost_model(list(range(remote_experts)), bytes_per_expert, link,
                                             prefetch_window_us=prefetch_window_us).critical_path_us
    rows = num_tokens * top_k
    remote_bytes = int(math.ceil(rows * (world_size - 1) / max(1, world_size))) * hidden_size * 2
    ep = local_layer_us + ep_exchange_us + 2 * link.copy_us(remote_bytes) if world_size > 1 else local_layer_us
    return DecodePathChoice("ep" if ep < dwdp else "dwdp", ep, dwdp)


def measure_link(store, experts_per_sample: tuple[int, ...] = (1, 4, 8), repeats: int = 5) -> LinkProfile:
    """Fit a LinkProfile from timed engine prefetches of 1, 4 and 8 remote experts of a connected
    ``ShardedExpertStore`` (CUDA events on the current stream, after warm-up). Batches of at
    least ``streams`` copies give the aggregate rate and the latency (their slope and
    intercept); the single copy then gives one stream's rate."""
    import torch

    if len(store.remote) < max(experts_per_sample):
        raise ValueError("the store has too few remote experts to time")
    streams = getattr(store.engine, "num_streams", 4)
    nbytes = store.slab_bytes
    samples = []
    for n in experts_per_sample:
        ids = store.remote[:n]
        for _ in range(2):
            store.engine.prefetch_into(ids, 0)
            store.engine.wait_buffer(0)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(repeats):
            store.engine.prefetch_into(ids, 0)
            store.engine.wait_buffer(0)
        b.record()
        torch.cuda.synchronize()
        samples.append((n, a.elapsed_time(b) * 1e3 / repeats))
    agg = fit_link([(k * nbytes, t) for k, t in samples if k >= streams], streams=1)
    single = [t for k, t in samples if k == 1]
    if single and single[0] > agg.latency_us:
        per_stream = nbytes / ((single[0] - agg.latency_us) * 1e3)
    else:
        per_stream = agg.bandwidth_gbps / streams
    return LinkProfile(latency_us=agg.latency_us, bandwidth_gbps=per_stream, aggregate_gbps=agg.bandwidth_gbps,
                       streams=streams)

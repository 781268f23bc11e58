"""Time model of a placement: compute per stage, transfers per boundary, step time.

* compute(flops on worker w)   = forward FLOPs x (1 + BACKWARD_FACTOR) / w.measured_flops
* boundary transfer            = host-staged: bytes/d2h(src) + latency + bytes/bandwidth + bytes/h2d(dst)
                                 NCCL over NVLink (GPUs of one box): latency + bytes / NVLink bandwidth
* stage time per microbatch    = compute + transfers, or max(compute, transfers) when transfers overlap
* step                         ~ (M + S - 1) x slowest stage time per microbatch

The same model as the reference's planner (planner/cost.py:1-83), with NVLink
device links added: NVLINK_P2P_BPS is the measured B200 peer-copy rate per
direction, and an unmeasured network link defaults to 1 ms and 100 Mbit/s.
"""

from __future__ import annotations

from dataclasses import dataclass, field

BACKWARD_FACTOR = 2.0
DEFAULT_LATENCY_S = 1e-3
DEFAULT_BANDWIDTH_BPS = 100e6 / 8
NVLINK_P2P_BPS = 770e9
NVLINK_LATENCY_S = 10e-6


@dataclass
class NetworkModel:
    """Directional per-pair link costs, keyed by (source worker id, destination worker id)."""

    latency: dict[tuple[str, str], float] = field(default_factory=dict)
    bandwidth: dict[tuple[str, str], float] = field(default_factory=dict)
    device_links: set[tuple[str, str]] = field(default_factory=set)  # NCCL over NVLink, no host staging

    def link(self, src: str, dst: str) -> tuple[float, float]:
        """(latency s, bandwidth B/s) of src -> dst; measured values win over defaults."""
        pair = (src, dst)
        if pair in self.device_links and pair not in self.bandwidth:
            return NVLINK_LATENCY_S, NVLINK_P2P_BPS
        return self.latency.get(pair, DEFAULT_LATENCY_S), self.bandwidth.get(pair, DEFAULT_BANDWIDTH_BPS)

    def transfer_time(self, nbytes: float, src: str, dst: str) -> float:
        if src == dst:
            return 0.0
        latency, bandwidth = self.link(src, dst)
        return latency + nbytes / bandwidth

    @classmethod
    def from_measurements(cls, links: dict[str, dict]) -> "NetworkModel":
        """``links``: {"src->dst": probe result} as produced by the cluster benchmark."""
        model = cls()
        for name, probe in links.items():
            pair = tuple(name.split("->"))
            model.latency[pair] = probe["latency_s"]
            model.bandwidth[pair] = probe["bandwidth_Bps"]
            if probe.get("kind") == "nccl":
                model.device_links.add(pair)
        return model


def compute_time(flops: float, measured_flops: float) -> float:
    """Forward plus backward seconds of ``flops`` forward FLOPs."""
    return flops * (1.0 + BACKWARD_FACTOR) / max(measured_flops, 1.0)


def pipeline_step_time(stage_times_per_mb: list[float], num_microbatches: int) -> float:
    if not stage_times_per_mb:
        return 0.0
    slowest = max(stage_times_per_mb)
    return (num_microbatches + len(stage_times_per_mb) - 1) * slowest


def boundary_transfer_time(nbytes: float, src, dst, network: NetworkModel) -> dict:
    """Seconds to move one boundary tensor from worker ``src`` to ``dst``, by phase."""
    wire = network.transfer_time(nbytes, src.worker_id, dst.worker_id)
    if (src.worker_id, dst.worker_id) in network.device_links:
        return {"d2h_s": 0.0, "network_s": wire, "h2d_s": 0.0, "total_s": wire, "kind": "nccl"}
    d2h = nbytes / src.d2h_Bps if src.d2h_Bps else 0.0
    h2d = nbytes / dst.h2d_Bps if dst.h2d_Bps else 0.0
    return {"d2h_s": d2h, "network_s": wire, "h2d_s": h2d, "total_s": d2h + wire + h2d, "kind": "host"}

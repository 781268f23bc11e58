"""Pipeline placement cost model (reference planner/cost.py:1-83, recalibrated for B200).

    network(bytes, i->j)  = latency[i][j] + bytes / bandwidth[i][j]
    transfer(bytes, i->j) = bytes / d2h[i] + network + bytes / h2d[j]      host-staged links (TCP)
                          = latency + bytes / nvlink_bw                     NCCL p2p between GPUs of one box
    compute(v, i)         = flops[v] * (1 + 2) / measured_flops[i]         (backward ~ 2x forward)
    stage_time            = compute + comm  (blocking)  |  max(compute, comm)  (async / NCCL streams)
    step                  ~= (M + S - 1) * max_s stage_time_s
"""

from __future__ import annotations

from dataclasses import dataclass, field

BACKWARD_FACTOR = 2.0
DEFAULT_LATENCY_S = 1e-3
DEFAULT_BANDWIDTH_BPS = 100e6 / 8        # unmeasured network link: 100 Mbit/s
NVLINK_P2P_BPS = 770e9                   # measured B200 peer copy, per direction
NVLINK_LATENCY_S = 10e-6


@dataclass
class NetworkModel:
    latency: dict[tuple[str, str], float] = field(default_factory=dict)
    bandwidth: dict[tuple[str, str], float] = field(default_factory=dict)
    # pairs connected by NCCL over NVLink inside one box (no host staging)
    device_links: set[tuple[str, str]] = field(default_factory=set)

    def transfer_time(self, nbytes: float, src: str, dst: str) -> float:
        if src == dst:
            return 0.0
        if (src, dst) in self.device_links and (src, dst) not in self.bandwidth:
            return NVLINK_LATENCY_S + nbytes / NVLINK_P2P_BPS
        return self.latency.get((src, dst), DEFAULT_LATENCY_S) + nbytes / self.bandwidth.get((src, dst),
                                                                                              DEFAULT_BANDWIDTH_BPS)

    @classmethod
    def from_measurements(cls, links: dict[str, dict]) -> "NetworkModel":
        nm = cls()
        for key, m in links.items():
            src, dst = key.split("->")
            nm.latency[(src, dst)] = m["latency_s"]
            nm.bandwidth[(src, dst)] = m["bandwidth_Bps"]
            if m.get("kind") == "nccl":
                nm.device_links.add((src, dst))
        return nm


def compute_time(flops: float, measured_flops: float) -> float:
    return flops * (1 + BACKWARD_FACTOR) / max(measured_flops, 1.0)


def pipeline_step_time(stage_times_per_mb: list[float], num_microbatches: int) -> float:
    if not stage_times_per_mb:
        return 0.0
    return (num_microbatches + len(stage_times_per_mb) - 1) * max(stage_times_per_mb)


def boundary_transfer_time(nbytes: float, src, dst, network: NetworkModel) -> dict:
    """``src``/``dst`` are WorkerProfiles; NCCL device links skip host staging."""
    if (src.worker_id, dst.worker_id) in network.device_links:
        net = network.transfer_time(nbytes, src.worker_id, dst.worker_id)
        return {"d2h_s": 0.0, "network_s": net, "h2d_s": 0.0, "total_s": net, "kind": "nccl"}
    d2h = nbytes / src.d2h_Bps if src.d2h_Bps else 0.0
    h2d = nbytes / dst.h2d_Bps if dst.h2d_Bps else 0.0
    net = network.transfer_time(nbytes, src.worker_id, dst.worker_id)
    return {"d2h_s": d2h, "network_s": net, "h2d_s": h2d, "total_s": d2h + net + h2d, "kind": "host"}

"""Emulated heterogeneous workers on one CPU host (reference experiments/emulation.py:1-47).

Each emulated worker is a separate CPU process with its own torch thread count
(a real, measured compute difference) and a declared memory budget (enforced by
the planner's accounting and checked against the bytes the stage really held).
Results produced this way are labelled "emulated".
"""

from __future__ import annotations

import multiprocessing as mp
from dataclasses import dataclass

from meshtrain_b200.planner.partition import WorkerProfile

MB = 1024 ** 2


@dataclass
class EmulatedWorker:
    name: str
    threads: int
    memory_budget_bytes: int
    label: str = ""


def _bench(threads: int) -> dict:
    import torch

    from meshtrain_b200.profiler.benchmark import benchmark_device
    from meshtrain_b200.worker.device import CPUDeviceAdapter

    torch.set_num_threads(threads)
    return benchmark_device(CPUDeviceAdapter(), matmul_size=768, iters=8)


def profile_emulated(workers: list[EmulatedWorker]) -> list[WorkerProfile]:
    """Benchmark every emulated worker in its own process, one after another (no core contention)."""
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:
        results = [pool.apply(_bench, (w.threads,)) for w in workers]
    best = max(r["measured_flops"] for r in results)
    return [WorkerProfile(w.name, w.name, "cpu", w.memory_budget_bytes, r["measured_flops"],
                          compute_score=r["measured_flops"] / best) for w, r in zip(workers, results)]

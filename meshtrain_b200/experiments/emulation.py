"""Heterogeneous workers emulated on one CPU host.

An emulated worker is a CPU process limited to a number of torch threads (a
real, measured difference in compute speed) with a declared memory budget
that the planner's accounting enforces.  ``profile_emulated`` measures each
one in a fresh process, one at a time so they do not compete for cores, and
returns planner profiles whose compute scores are relative to the fastest.
The experiments that use these label their results "emulated" (the role of
the reference's emulated workers, experiments/emulation.py:1-47).
"""

from __future__ import annotations

from concurrent.futures import ProcessPoolExecutor
from dataclasses import dataclass
import multiprocessing as mp

from meshtrain_b200.planner.partition import WorkerProfile

MB = 1024 ** 2


@dataclass
class EmulatedWorker:
    name: str
    threads: int
    memory_budget_bytes: int
    label: str = ""


def _measure(threads: int) -> float:
    """FLOP/s of a CPU process limited to ``threads`` torch threads."""
    import torch

    from meshtrain_b200.profiler.benchmark import benchmark_device
    from meshtrain_b200.worker.device import CPUDeviceAdapter

    torch.set_num_threads(threads)
    return float(benchmark_device(CPUDeviceAdapter(), matmul_size=768, iters=8)["measured_flops"])


def profile_emulated(workers: list[EmulatedWorker]) -> list[WorkerProfile]:
    rates = []
    with ProcessPoolExecutor(max_workers=1, mp_context=mp.get_context("spawn")) as pool:
        for worker in workers:  # sequentially: no two measurements share the cores
            rates.append(pool.submit(_measure, worker.threads).result())
    fastest = max(rates)
    return [WorkerProfile(w.name, w.name, "cpu", w.memory_budget_bytes, rate, compute_score=rate / fastest)
            for w, rate in zip(workers, rates)]

"""Device micro-benchmarks feeding the planner.

Measures what the reference's worker benchmark reports (profiler/benchmark.py:32-97):
fp32 matmul GFLOP/s, an MLP forward and forward+backward, and 4 MiB host-to-device /
device-to-host copy rates. On CUDA devices it also measures the bf16 throughput
of this package's tcgen05 GEMM, which is the rate the device engine runs at.
``normalise_scores`` turns each worker's measured FLOP/s into a compute score
relative to the fastest worker.

Each workload is timed by ``_Clock``: CUDA events on the device's current stream
for a CUDA device (device time, no host jitter), ``perf_counter`` around a
synchronise elsewhere; the median of the repetitions is reported.
"""

from __future__ import annotations

import statistics
import time

import torch
from torch import nn

COPY_BYTES = 4 * 1024 * 1024
# Fraction of a bare GEMM's rate that a whole training step of the device engine reaches;
# the planner compares workers by step throughput, not by a single kernel.
ENGINE_STEP_EFFICIENCY = 0.7


class _Clock:
    def __init__(self, adapter):
        self.adapter = adapter
        self.device_timed = adapter.backend == "cuda"

    def median_s(self, fn, warmup: int, reps: int) -> float:
        for _ in range(warmup):
            fn()
        self.adapter.synchronize()
        if self.device_timed:
            marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                     for _ in range(reps)]
            stream = torch.cuda.current_stream(self.adapter.device)
            for begin, end in marks:
                begin.record(stream)
                fn()
                end.record(stream)
            self.adapter.synchronize()
            return statistics.median(b.elapsed_time(e) * 1e-3 for b, e in marks)
        laps = []
        for _ in range(reps):
            start = time.perf_counter()
            fn()
            self.adapter.synchronize()
            laps.append(time.perf_counter() - start)
        return statistics.median(laps)


def _mlp(width: int, depth: int = 3) -> nn.Sequential:
    mods: list[nn.Module] = []
    for i in range(depth):
        mods.append(nn.Linear(width, width))
        if i + 1 < depth:
            mods.append(nn.GELU())
    return nn.Sequential(*mods)


def _tcgen05_tflops(adapter, n: int = 4096, reps: int = 10) -> float | None:
    """bf16 TFLOP/s of the package's own GEMM on an n x n x n problem (None off CUDA)."""
    from meshtrain_b200 import ops

    if adapter.backend != "cuda" or not ops.extension_available():
        return None
    a = torch.randn(n, n, device=adapter.device, dtype=torch.bfloat16)
    b = torch.randn(n, n, device=adapter.device, dtype=torch.bfloat16)
    per_call = _Clock(adapter).median_s(lambda: ops.linear(a, b), 3, reps)
    return 2.0 * n ** 3 / per_call / 1e12


def benchmark_device(adapter, *, matmul_size: int = 1024, iters: int = 10, mlp_batch: int = 64,
                     mlp_hidden: int = 1024, quick: bool = False) -> dict:
    if quick:
        matmul_size, iters, mlp_hidden = 512, 3, 512
    clock = _Clock(adapter)
    gen = torch.Generator().manual_seed(0)
    lhs, rhs = (adapter.move_tensor(torch.randn(matmul_size, matmul_size, generator=gen)) for _ in range(2))
    matmul_s = clock.median_s(lambda: torch.mm(lhs, rhs), 2, iters)
    gflops = 2.0 * matmul_size ** 3 / matmul_s / 1e9

    with torch.random.fork_rng(devices=[]):  # same weights on every worker, caller's RNG untouched
        torch.manual_seed(0)
        net = _mlp(mlp_hidden)
    net = adapter.move_module(net)
    batch = adapter.move_tensor(torch.randn(mlp_batch, mlp_hidden, generator=gen))

    def forward_only():
        with torch.no_grad():
            net(batch)

    def forward_backward():
        net(batch).sum().backward()

    fwd_s = clock.median_s(forward_only, 2, iters)
    fwd_bwd_s = clock.median_s(forward_backward, 2, iters)

    on_host = adapter.backend == "cpu"
    staged = torch.randn(COPY_BYTES // 4)
    if adapter.backend == "cuda":
        staged = staged.pin_memory()
    resident = adapter.move_tensor(staged)
    copy_reps = max(3, iters // 2)
    h2d_s = clock.median_s(lambda: adapter.move_tensor(staged), 1, copy_reps)
    d2h_s = clock.median_s(lambda: resident.to("cpu"), 1, copy_reps)

    def gbps(seconds: float) -> float:
        return COPY_BYTES / seconds / 1e9 if seconds > 0 else float("inf")

    report = {
        "backend": adapter.backend, "device": str(adapter.device), "device_name": adapter.name(),
        "matmul_size": matmul_size, "matmul_s": matmul_s, "matmul_gflops": gflops,
        "mlp_forward_s": fwd_s, "mlp_backward_s": max(0.0, fwd_bwd_s - fwd_s), "mlp_fwd_bwd_s": fwd_bwd_s,
        "host_to_device_GBps": gbps(h2d_s), "device_to_host_GBps": gbps(d2h_s),
        # a CPU worker copies nothing across a bus; the planner reads 0 as "no staging cost"
        "h2d_Bps": 0.0 if on_host else COPY_BYTES / max(h2d_s, 1e-9),
        "d2h_Bps": 0.0 if on_host else COPY_BYTES / max(d2h_s, 1e-9),
        "measured_flops": gflops * 1e9,
    }
    if not quick:
        tflops = _tcgen05_tflops(adapter)
        if tflops:
            report["bf16_gemm_tflops"] = tflops
            report["measured_flops"] = tflops * 1e12 * ENGINE_STEP_EFFICIENCY
    return report


def normalise_scores(benchmarks: dict[str, dict]) -> dict[str, float]:
    """Each worker's measured FLOP/s divided by the fastest worker's."""
    rates = {worker: float(b["measured_flops"]) for worker, b in benchmarks.items()}
    top = max(rates.values(), default=0.0)
    return {worker: rate / top for worker, rate in rates.items()} if top > 0 else dict.fromkeys(rates, 0.0)

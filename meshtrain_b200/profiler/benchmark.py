"""Device micro-benchmarks feeding the planner (reference profiler/benchmark.py:32-97).

Measures fp32 matmul GFLOP/s, an MLP forward/backward, 4 MB H2D/D2H rates,
and on CUDA devices also the bf16 throughput of this package's tcgen05 GEMM
(the number the GPU engine actually runs at).  ``compute_score`` is each
worker's measured FLOP/s relative to the fastest worker.
"""

from __future__ import annotations

import statistics
import time

import torch
from torch import nn


def _timeit(fn, adapter, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    adapter.synchronize()
    samples = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        adapter.synchronize()
        samples.append(time.perf_counter() - t0)
    return statistics.median(samples)


def _cuda_gemm_tflops(adapter, n: int = 4096, iters: int = 10) -> float | None:
    from meshtrain_b200 import ops

    if adapter.backend != "cuda" or not ops.extension_available():
        return None
    dev = adapter.device
    a = torch.randn(n, n, device=dev).to(torch.bfloat16)
    b = torch.randn(n, n, device=dev).to(torch.bfloat16)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        ops.linear(a, b)
    s.record()
    for _ in range(iters):
        ops.linear(a, b)
    e.record()
    e.synchronize()
    return 2 * n ** 3 * iters / (s.elapsed_time(e) / 1e3) / 1e12


def benchmark_device(adapter, *, matmul_size: int = 1024, iters: int = 10, mlp_batch: int = 64,
                     mlp_hidden: int = 1024, quick: bool = False) -> dict:
    if quick:
        matmul_size, iters, mlp_hidden = 512, 3, 512
    g = torch.Generator().manual_seed(0)
    a = adapter.move_tensor(torch.randn(matmul_size, matmul_size, generator=g))
    b = adapter.move_tensor(torch.randn(matmul_size, matmul_size, generator=g))
    mm_s = _timeit(lambda: a @ b, adapter, 2, iters)
    gflops = 2 * matmul_size ** 3 / mm_s / 1e9
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(0)
        mlp = nn.Sequential(nn.Linear(mlp_hidden, mlp_hidden), nn.GELU(), nn.Linear(mlp_hidden, mlp_hidden), nn.GELU(),
                            nn.Linear(mlp_hidden, mlp_hidden))
    mlp = adapter.move_module(mlp)
    x = adapter.move_tensor(torch.randn(mlp_batch, mlp_hidden, generator=g))

    def fwd():
        with torch.no_grad():
            mlp(x)

    def fwd_bwd():
        mlp(x).sum().backward()

    fwd_s = _timeit(fwd, adapter, 2, iters)
    fb_s = _timeit(fwd_bwd, adapter, 2, iters)
    host = torch.randn(1024 * 1024)  # 4 MB
    if adapter.backend == "cuda":
        host = host.pin_memory()
    h2d_s = _timeit(lambda: adapter.move_tensor(host), adapter, 1, max(3, iters // 2))
    dev_t = adapter.move_tensor(host)
    d2h_s = _timeit(lambda: dev_t.to("cpu"), adapter, 1, max(3, iters // 2))
    nbytes = host.numel() * 4
    on_host = adapter.backend == "cpu"
    out = {"backend": adapter.backend, "device": str(adapter.device), "device_name": adapter.name(),
           "matmul_size": matmul_size, "matmul_s": mm_s, "matmul_gflops": gflops, "mlp_forward_s": fwd_s,
           "mlp_backward_s": max(fb_s - fwd_s, 0.0), "mlp_fwd_bwd_s": fb_s,
           "host_to_device_GBps": nbytes / h2d_s / 1e9 if h2d_s > 0 else float("inf"),
           "device_to_host_GBps": nbytes / d2h_s / 1e9 if d2h_s > 0 else float("inf"),
           "h2d_Bps": 0.0 if on_host else nbytes / max(h2d_s, 1e-9),
           "d2h_Bps": 0.0 if on_host else nbytes / max(d2h_s, 1e-9),
           "measured_flops": gflops * 1e9}
    if not quick:
        tc = _cuda_gemm_tflops(adapter)
        if tc:
            out["bf16_gemm_tflops"] = tc
            out["measured_flops"] = tc * 1e12 * 0.7  # whole-step efficiency of the engine vs a bare GEMM
    return out


def normalise_scores(benchmarks: dict[str, dict]) -> dict[str, float]:
    if not benchmarks:
        return {}
    best = max(b["measured_flops"] for b in benchmarks.values())
    return {w: b["measured_flops"] / best for w, b in benchmarks.items()}

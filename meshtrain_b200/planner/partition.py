"""Contiguous-layer placement planner (reference planner/partition.py:36-395).

Strategies:
  equal            same number of layers per worker, in the given order
  compute          contiguous split with each worker's share of FLOPs proportional to its speed
  auto / topology_aware
                   for each ordered subset of eligible workers (at most ``max_orderings``),
                   an exact DP over contiguous splits minimising the bottleneck stage time
                   (compute + boundary transfers) under every worker's memory budget; within
                   ``tie_tolerance`` it prefers fewer boundary bytes, then fewer stages
  manual           explicit (worker, start, end) assignments
Every plan is memory-checked; equal/compute report violations instead of overcommitting.
"""

from __future__ import annotations

import itertools
import math
from dataclasses import dataclass, field

from meshtrain_b200.planner.cost import NetworkModel, boundary_transfer_time, compute_time, pipeline_step_time
from meshtrain_b200.planner.graph import LayerProfile
from meshtrain_b200.planner.memory import (DEFAULT_FRAMEWORK_RESERVE, DEFAULT_SAFETY_FACTOR, MemoryEstimate,
                                           estimate_stage_memory, reserved_bytes)


@dataclass
class WorkerProfile:
    worker_id: str
    name: str
    backend: str
    memory_total: int
    measured_flops: float
    unified_memory: bool = False
    supported_dtypes: tuple[str, ...] = ("float32", "float16", "bfloat16", "float64")
    compute_score: float = 1.0
    supported_ops: dict | None = None
    d2h_Bps: float = 0.0
    h2d_Bps: float = 0.0
    memory_available: int | None = None
    host: str | None = None  # GPUs of one host are linked by NCCL over NVLink


@dataclass
class StagePlan:
    stage_index: int
    worker_id: str
    worker_name: str
    backend: str
    start: int
    end: int
    memory: MemoryEstimate
    compute_s: float
    comm_s: float
    boundary_bytes: int
    overlap: bool = False
    comm_detail: dict = field(default_factory=dict)

    @property
    def time_per_mb(self) -> float:
        return max(self.compute_s, self.comm_s) if self.overlap else self.compute_s + self.comm_s


@dataclass
class Plan:
    strategy: str
    stages: list[StagePlan]
    num_microbatches: int
    excluded: dict[str, str] = field(default_factory=dict)
    violations: list[str] = field(default_factory=list)

    @property
    def feasible(self) -> bool:
        return bool(self.stages) and not self.violations

    @property
    def bottleneck(self) -> StagePlan | None:
        return max(self.stages, key=lambda s: s.time_per_mb) if self.stages else None

    @property
    def predicted_step_s(self) -> float:
        return pipeline_step_time([s.time_per_mb for s in self.stages], self.num_microbatches)

    @property
    def communication_bytes_per_step(self) -> int:
        return sum(2 * self.num_microbatches * s.boundary_bytes for s in self.stages[:-1])

    @property
    def communication_s_per_step(self) -> float:
        return sum(self.num_microbatches * s.comm_s for s in self.stages)

    def ranges(self) -> list[tuple[int, int]]:
        return [(s.start, s.end) for s in self.stages]

    def boundaries(self) -> list[dict]:
        return [{"from_stage": a.stage_index, "to_stage": b.stage_index, "activation_bytes": a.boundary_bytes,
                 "gradient_bytes": a.boundary_bytes, "forward": a.comm_detail.get("forward", {}),
                 "backward": b.comm_detail.get("backward", {})} for a, b in zip(self.stages, self.stages[1:])]

    def to_dict(self) -> dict:
        return {"boundaries": self.boundaries(), "strategy": self.strategy, "feasible": self.feasible,
                "violations": self.violations, "excluded": self.excluded, "num_microbatches": self.num_microbatches,
                "predicted_step_s": self.predicted_step_s,
                "communication_bytes_per_step": self.communication_bytes_per_step,
                "communication_s_per_step": self.communication_s_per_step,
                "stages": [{"stage": s.stage_index, "worker_id": s.worker_id, "worker": s.worker_name,
                            "backend": s.backend, "layers": [s.start, s.end], "compute_s_per_mb": s.compute_s,
                            "comm_s_per_mb": s.comm_s, "time_per_mb": s.time_per_mb, "overlap": s.overlap,
                            "boundary_bytes": s.boundary_bytes, "memory": s.memory.to_dict()} for s in self.stages]}

    def format(self, layer_names: list[str] | None = None) -> str:
        gb = lambda n: f"{n / 1024 ** 3:.2f} GB"  # noqa: E731
        lines = [f"Proposed placement ({self.strategy}):", ""]
        for s in self.stages:
            names = f" ({layer_names[s.start]} .. {layer_names[s.end - 1]})" if layer_names else ""
            lines += [f"  Stage {s.stage_index} -> {s.worker_name} [{s.backend}]",
                      f"      layers {s.start}-{s.end - 1}{names}",
                      f"      memory {gb(s.memory.required)} of {gb(s.memory.budget)} usable"
                      f" ({'ok' if s.memory.fits else 'OVER BUDGET'})",
                      f"      compute {s.compute_s * 1000:.2f} ms/mb, send {s.comm_s * 1000:.2f} ms/mb"]
        b = self.bottleneck
        lines += ["", "Predicted:",
                  f"  communication/step: {self.communication_bytes_per_step / 1e6:.2f} MB "
                  f"({self.communication_s_per_step * 1000:.1f} ms)"]
        if b:
            lines.append(f"  slowest stage: {b.stage_index} ({b.worker_name}, {b.time_per_mb * 1000:.2f} ms/mb)")
        lines.append(f"  estimated pipeline time: {self.predicted_step_s * 1000:.1f} ms/step "
                     f"(M={self.num_microbatches}, S={len(self.stages)})")
        if self.excluded:
            lines.append("  excluded workers: " + ", ".join(f"{w} ({why})" for w, why in self.excluded.items()))
        lines += [f"  VIOLATION: {v}" for v in self.violations]
        return "\n".join(lines)


@dataclass
class PlannerOptions:
    optimizer: str = "sgd"
    num_microbatches: int = 1
    allow_backends: tuple[str, ...] = ("cuda", "mps", "cpu")
    dtype: str = "float32"
    headroom_fraction: float | None = None
    headroom_min_bytes: int | None = None
    activation_safety: float = 1.25
    num_stages: int | None = None
    max_orderings: int = 400
    schedule: str = "gpipe"
    max_inflight: int | None = None
    safety_factors: dict = field(default_factory=lambda: dict(DEFAULT_SAFETY_FACTOR))
    framework_reserve: dict = field(default_factory=lambda: dict(DEFAULT_FRAMEWORK_RESERVE))
    budget_overrides: dict = field(default_factory=dict)
    required_ops: tuple[str, ...] = ()
    async_transport: bool = False
    tie_tolerance: float = 0.02
    engine: str = "autograd"          # "device": GPU engine memory accounting
    param_dtype_bytes: int = 4
    offload: bool = False

    def memory_kwargs(self, backend: str) -> dict:
        if self.headroom_fraction is not None or self.headroom_min_bytes is not None:
            return {"headroom_fraction": self.headroom_fraction, "headroom_min_bytes": self.headroom_min_bytes}
        return {"safety_factor": self.safety_factors.get(backend, 0.85),
                "framework_reserve": self.framework_reserve.get(backend, 0)}


class _Evaluator:
    def __init__(self, layers: list[LayerProfile], network: NetworkModel, opts: PlannerOptions):
        self.layers, self.network, self.opts = layers, network, opts
        self.prefix = list(itertools.accumulate((l.flops for l in layers), initial=0.0))
        self._cache: dict = {}

    def stage(self, idx: int, ws: list[WorkerProfile], start: int, end: int) -> StagePlan:
        key = (idx, tuple(w.worker_id for w in ws[max(0, idx - 1):idx + 2]), len(ws), start, end)
        if key in self._cache:
            return self._cache[key]
        w = ws[idx]
        last = idx == len(ws) - 1
        comp = compute_time(self.prefix[end] - self.prefix[start], w.measured_flops)
        out_bytes = 0 if last else self.layers[end - 1].activation_bytes
        comm, detail = 0.0, {}
        if not last:
            detail["forward"] = boundary_transfer_time(out_bytes, w, ws[idx + 1], self.network)
            comm += detail["forward"]["total_s"]
        if idx > 0:
            detail["backward"] = boundary_transfer_time(self.layers[start].input_bytes, w, ws[idx - 1], self.network)
            comm += detail["backward"]["total_s"]
        total = self.opts.budget_overrides.get(w.worker_id, w.memory_total)
        mem = estimate_stage_memory(self.layers[start:end], total=total, optimizer=self.opts.optimizer,
                                    num_microbatches=self.opts.num_microbatches, is_last=last, stage_index=idx,
                                    num_stages=len(ws), schedule=self.opts.schedule,
                                    max_inflight=self.opts.max_inflight, backend=w.backend,
                                    activation_safety=self.opts.activation_safety, available=w.memory_available,
                                    engine=self.opts.engine, param_dtype_bytes=self.opts.param_dtype_bytes,
                                    offload=self.opts.offload, **self.opts.memory_kwargs(w.backend))
        sp = StagePlan(idx, w.worker_id, w.name, w.backend, start, end, mem, comp, comm, out_bytes,
                       overlap=self.opts.async_transport, comm_detail=detail)
        self._cache[key] = sp
        return sp


def _usable(w: WorkerProfile, opts: PlannerOptions) -> int:
    total = opts.budget_overrides.get(w.worker_id, w.memory_total)
    kw = opts.memory_kwargs(w.backend)
    if "headroom_fraction" in kw:
        usable = total - reserved_bytes(total, kw["headroom_fraction"] or 0.0, kw["headroom_min_bytes"] or 0)
    else:
        usable = int(total * kw["safety_factor"]) - kw["framework_reserve"]
    return usable if w.memory_available is None else min(usable, w.memory_available)


def eligible_workers(workers: list[WorkerProfile], opts: PlannerOptions):
    ok, excluded = [], {}
    for w in workers:
        missing = []
        if w.supported_ops is not None:
            missing = sorted(set(opts.required_ops) - set(w.supported_ops.get(opts.dtype, ())))
        if w.backend not in opts.allow_backends:
            excluded[w.name] = f"backend {w.backend} not allowed"
        elif opts.dtype not in w.supported_dtypes:
            excluded[w.name] = f"no {opts.dtype} support"
        elif missing:
            excluded[w.name] = f"cannot run {', '.join(missing)} in {opts.dtype}"
        elif _usable(w, opts) <= 0:
            excluded[w.name] = "memory below safety margin"
        else:
            ok.append(w)
    return ok, excluded


def _checked(plan: Plan, n_layers: int) -> Plan:
    sizes = [s.end - s.start for s in plan.stages]
    if sum(sizes) != n_layers or any(c <= 0 for c in sizes):
        plan.violations.append("partition does not cover every layer exactly once")
    for s in plan.stages:
        if not s.memory.fits:
            plan.violations.append(f"stage {s.stage_index} on {s.worker_name} needs "
                                   f"{s.memory.required / 1024 ** 3:.2f} GB but only "
                                   f"{s.memory.budget / 1024 ** 3:.2f} GB is usable")
    return plan


def _from_bounds(strategy, ws, bounds, ev, excluded) -> Plan:
    plan = Plan(strategy, [ev.stage(i, ws, a, b) for i, (a, b) in enumerate(bounds)], ev.opts.num_microbatches,
                excluded=dict(excluded))
    return _checked(plan, len(ev.layers))


def split_by_weights(n_layers: int, weights: list[float], layer_cost: list[float]) -> list[tuple[int, int]]:
    """Contiguous split whose cumulative layer cost tracks the cumulative weight share."""
    k = len(weights)
    costs = layer_cost if sum(layer_cost) > 0 else [1.0] * n_layers
    total = sum(costs)
    share = list(itertools.accumulate(w / sum(weights) for w in weights))
    bounds, start, acc = [], 0, 0.0
    for i in range(k):
        if i == k - 1:
            end = n_layers
        else:
            target = share[i] * total
            end = start + 1
            acc += costs[start]
            while end < n_layers - (k - 1 - i) and acc + costs[end] / 2 <= target:
                acc += costs[end]
                end += 1
        bounds.append((start, end))
        start = end
    return bounds


def plan_equal(layers, workers, network, opts) -> Plan:
    ws, excluded = eligible_workers(workers, opts)
    k = min(opts.num_stages or len(ws), len(ws), len(layers))
    n = len(layers)
    return _from_bounds("equal", ws[:k], [(n * i // k, n * (i + 1) // k) for i in range(k)],
                        _Evaluator(layers, network, opts), excluded)


def plan_compute(layers, workers, network, opts) -> Plan:
    ws, excluded = eligible_workers(workers, opts)
    k = min(opts.num_stages or len(ws), len(ws), len(layers))
    chosen = sorted(ws, key=lambda w: -w.measured_flops)[:k]
    ws = [w for w in workers if w in chosen]
    bounds = split_by_weights(len(layers), [w.measured_flops for w in ws], [max(l.flops, 1.0) for l in layers])
    return _from_bounds("compute", ws, bounds, _Evaluator(layers, network, opts), excluded)


def _better(a, b, tol: float) -> bool:
    """(bottleneck, bytes): clearly faster wins; within tol, fewer boundary bytes wins."""
    if b[0] == math.inf:
        return a[0] < math.inf
    if a[0] < b[0] * (1 - tol):
        return True
    return a[0] <= b[0] * (1 + tol) and a[1] < b[1]


def _dp(ev: _Evaluator, ws: list[WorkerProfile]):
    n, k = len(ev.layers), len(ws)
    inf = (math.inf, math.inf, None)
    best = [[inf] * (k + 1) for _ in range(n + 1)]
    best[0][0] = (0.0, 0.0, None)
    for s in range(1, k + 1):
        for j in range(s, n - (k - s) + 1):
            cand = inf
            for i in range(s - 1, j):
                prev = best[i][s - 1]
                if prev[0] == math.inf:
                    continue
                st = ev.stage(s - 1, ws, i, j)
                if not st.memory.fits:
                    continue
                val = (max(prev[0], st.time_per_mb), prev[1] + st.boundary_bytes, i)
                if _better(val, cand, ev.opts.tie_tolerance):
                    cand = val
            best[j][s] = cand
    if best[n][k][0] == math.inf:
        return None
    bounds, j = [], n
    for s in range(k, 0, -1):
        i = best[j][s][2]
        bounds.append((i, j))
        j = i
    return best[n][k][:2], bounds[::-1]


def _signature(w: WorkerProfile) -> tuple:
    return (w.backend, w.memory_total, w.measured_flops, w.host, w.d2h_Bps, w.h2d_Bps, w.memory_available,
            w.unified_memory)


def _orderings(ws: list[WorkerProfile], k: int, network: NetworkModel):
    """Ordered k-subsets, skipping orderings that only swap interchangeable workers
    (same profile, same links to everyone) - e.g. the GPUs of one box."""
    seen = set()
    ids = [w.worker_id for w in ws]

    def link_sig(w):
        return tuple(sorted((network.latency.get((w.worker_id, o)), network.bandwidth.get((w.worker_id, o)),
                             (w.worker_id, o) in network.device_links) for o in ids if o != w.worker_id))

    sig = {w.worker_id: (_signature(w), link_sig(w)) for w in ws}
    for order in itertools.permutations(ws, k):
        key = tuple(sig[w.worker_id] for w in order)
        if key in seen:
            continue
        seen.add(key)
        yield order


def plan_auto(layers, workers, network, opts) -> Plan:
    ws, excluded = eligible_workers(workers, opts)
    ev = _Evaluator(layers, network, opts)
    sizes = [opts.num_stages] if opts.num_stages else range(1, min(len(ws), len(layers)) + 1)
    best = None
    tried = 0
    for k in sizes:
        for order in _orderings(ws, k, network):
            tried += 1
            if tried > opts.max_orderings:
                break
            res = _dp(ev, list(order))
            if res is None:
                continue
            key, bounds = res
            if best is None or key[0] < best[0][0] * 0.98 or (
                    abs(key[0] - best[0][0]) <= best[0][0] * 0.02 and (k, key[1]) < (len(best[1]), best[0][1])):
                best = (key, list(order), bounds)
    if best is None:
        plan = Plan("auto", [], opts.num_microbatches, excluded=excluded)
        plan.violations.append("no contiguous partition fits the memory budgets of the eligible workers")
        return plan
    _, order, bounds = best
    return _from_bounds("auto", order, bounds, ev, excluded)


def plan_manual(layers, workers, network, opts, assignments: list[tuple[str, int, int]]) -> Plan:
    by = {w.worker_id: w for w in workers} | {w.name: w for w in workers}
    ws = []
    for wid, _a, _b in assignments:
        if wid not in by:
            raise ValueError(f"manual placement names unknown worker {wid!r}")
        ws.append(by[wid])
    return _from_bounds("manual", ws, [(a, b) for _, a, b in assignments], _Evaluator(layers, network, opts), {})


STRATEGIES = {"equal": plan_equal, "compute": plan_compute, "auto": plan_auto, "topology_aware": plan_auto}


def make_plan(strategy: str, layers, workers, network: NetworkModel | None = None,
              opts: PlannerOptions | None = None) -> Plan:
    if strategy not in STRATEGIES:
        raise ValueError(f"unknown strategy {strategy!r}")
    return STRATEGIES[strategy](layers, workers, network or NetworkModel(), opts or PlannerOptions())


def b200_box(num_gpus: int = 8, memory_gb: float = 180.0, tflops: float = 1.2e15, host: str = "b200-box"):
    """Worker profiles + network model for one 8 x B200 NVLink box (NCCL links between every pair)."""
    ws = [WorkerProfile(f"{host}:gpu{i}", f"gpu{i}", "cuda", int(memory_gb * 1024 ** 3), tflops, host=host,
                        d2h_Bps=55e9, h2d_Bps=55e9) for i in range(num_gpus)]
    nm = NetworkModel()
    for a in ws:
        for b in ws:
            if a is not b:
                nm.device_links.add((a.worker_id, b.worker_id))
    return ws, nm

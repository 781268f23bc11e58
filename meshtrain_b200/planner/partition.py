"""Placement of contiguous layer ranges onto workers.

Strategies (the reference's, planner/partition.py:36-395):

* ``equal``: the same number of layers on each worker, in the given order.
* ``compute``: contiguous ranges whose FLOP shares follow the workers'
  measured FLOP rates; each cut sits at the layer boundary whose cumulative
  cost is nearest the cumulative rate share.
* ``auto`` / ``topology_aware``: for each ordered choice of workers, an exact
  search over the cut positions minimises the slowest stage's time per
  microbatch (compute plus its boundary transfers, overlapped or not) under
  every worker's memory budget; between candidates within ``tie_tolerance``
  (2 %) it prefers fewer boundary bytes, then fewer stages.  Orderings that
  only swap interchangeable workers (same profile and links, e.g. the GPUs of
  one NVSwitch box) are searched once.
* ``manual``: explicit (worker, start, end) assignments.

Every plan is memory-checked; ``equal`` / ``compute`` / ``manual`` report
violations instead of over-committing a device.
"""

from __future__ import annotations

import itertools
import math
from dataclasses import dataclass, field
from functools import lru_cache

from meshtrain_b200.planner.cost import NetworkModel, boundary_transfer_time, compute_time, pipeline_step_time
from meshtrain_b200.planner.graph import LayerProfile
from meshtrain_b200.planner.memory import (DEFAULT_FRAMEWORK_RESERVE, DEFAULT_SAFETY_FACTOR, MemoryEstimate,
                                           estimate_stage_memory, usable_bytes)

GB = 1024 ** 3


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
        return max(self.stages, key=lambda s: s.time_per_mb, default=None)

    @property
    def predicted_step_s(self) -> float:
        return pipeline_step_time([s.time_per_mb for s in self.stages], self.num_microbatches)

    @property
    def communication_bytes_per_step(self) -> int:
        # every boundary carries M activations forward and M gradients back
        return 2 * self.num_microbatches * sum(s.boundary_bytes for s in self.stages[:-1])

    @property
    def communication_s_per_step(self) -> float:
        return self.num_microbatches * sum(s.comm_s for s in self.stages)

    def ranges(self) -> list[tuple[int, int]]:
        return [(s.start, s.end) for s in self.stages]

    def boundaries(self) -> list[dict]:
        out = []
        for left, right in zip(self.stages, self.stages[1:]):
            out.append({"from_stage": left.stage_index, "to_stage": right.stage_index,
                        "activation_bytes": left.boundary_bytes, "gradient_bytes": left.boundary_bytes,
                        "forward": left.comm_detail.get("forward", {}),
                        "backward": right.comm_detail.get("backward", {})})
        return out

    def to_dict(self) -> dict:
        stages = [{"stage": s.stage_index, "worker_id": s.worker_id, "worker": s.worker_name, "backend": s.backend,
                   "layers": [s.start, s.end], "compute_s_per_mb": s.compute_s, "comm_s_per_mb": s.comm_s,
                   "time_per_mb": s.time_per_mb, "overlap": s.overlap, "boundary_bytes": s.boundary_bytes,
                   "memory": s.memory.to_dict()} for s in self.stages]
        return {"boundaries": self.boundaries(), "strategy": self.strategy, "feasible": self.feasible,
                "violations": self.violations, "excluded": self.excluded, "num_microbatches": self.num_microbatches,
                "predicted_step_s": self.predicted_step_s,
                "communication_bytes_per_step": self.communication_bytes_per_step,
                "communication_s_per_step": self.communication_s_per_step, "stages": stages}

    def format(self, layer_names: list[str] | None = None) -> str:
        text = [f"Proposed placement ({self.strategy}):", ""]
        for s in self.stages:
            span = f" ({layer_names[s.start]} .. {layer_names[s.end - 1]})" if layer_names else ""
            state = "ok" if s.memory.fits else "OVER BUDGET"
            text += [f"  Stage {s.stage_index} -> {s.worker_name} [{s.backend}]",
                     f"      layers {s.start}-{s.end - 1}{span}",
                     f"      memory {s.memory.required / GB:.2f} GB of {s.memory.budget / GB:.2f} GB usable ({state})",
                     f"      compute {s.compute_s * 1000:.2f} ms/mb, send {s.comm_s * 1000:.2f} ms/mb"]
        text += ["", "Predicted:", f"  communication/step: {self.communication_bytes_per_step / 1e6:.2f} MB "
                                   f"({self.communication_s_per_step * 1000:.1f} ms)"]
        slow = self.bottleneck
        if slow is not None:
            text.append(f"  slowest stage: {slow.stage_index} ({slow.worker_name}, {slow.time_per_mb * 1000:.2f} ms/mb)")
        text.append(f"  estimated pipeline time: {self.predicted_step_s * 1000:.1f} ms/step "
                    f"(M={self.num_microbatches}, S={len(self.stages)})")
        if self.excluded:
            text.append("  excluded workers: " + ", ".join(f"{w} ({why})" for w, why in self.excluded.items()))
        text += [f"  VIOLATION: {v}" for v in self.violations]
        return "\n".join(text)


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
    budget_overrides: dict = field(default_factory=dict)   # worker id -> total bytes (startup replanning)
    required_ops: tuple[str, ...] = ()
    async_transport: bool = False
    tie_tolerance: float = 0.02
    engine: str = "autograd"          # "device": GPU engine memory accounting
    param_dtype_bytes: int = 4
    offload: bool = False
    offload_ring: dict | None = None  # HostOffload settings (chunk_mb, device_budget_gb, ...) for the slot ring

    def memory_kwargs(self, backend: str) -> dict:
        if self.headroom_fraction is not None or self.headroom_min_bytes is not None:
            return {"headroom_fraction": self.headroom_fraction, "headroom_min_bytes": self.headroom_min_bytes}
        return {"safety_factor": self.safety_factors.get(backend, 0.85),
                "framework_reserve": self.framework_reserve.get(backend, 0)}

    def device_total(self, worker: WorkerProfile) -> int:
        return self.budget_overrides.get(worker.worker_id, worker.memory_total)


class StageCoster:
    """Prices layers [start, end) as stage ``index`` of a worker ordering (memoised)."""

    def __init__(self, layers: list[LayerProfile], network: NetworkModel, opts: PlannerOptions):
        self.layers, self.network, self.opts = layers, network, opts
        self.flops_before = list(itertools.accumulate((layer.flops for layer in layers), initial=0.0))
        self._memo: dict = {}

    def __call__(self, order: list[WorkerProfile], index: int, start: int, end: int) -> StagePlan:
        # a stage's price depends on its worker, its neighbours and the number of stages
        key = (tuple(w.worker_id for w in order[max(0, index - 1):index + 2]), index, len(order), start, end)
        plan = self._memo.get(key)
        if plan is None:
            plan = self._memo[key] = self._price(order, index, start, end)
        return plan

    def _price(self, order, index, start, end) -> StagePlan:
        opts, worker = self.opts, order[index]
        last = index == len(order) - 1
        detail = {}
        if not last:
            detail["forward"] = boundary_transfer_time(self.layers[end - 1].activation_bytes, worker,
                                                       order[index + 1], self.network)
        if index > 0:
            detail["backward"] = boundary_transfer_time(self.layers[start].input_bytes, worker, order[index - 1],
                                                        self.network)
        memory = estimate_stage_memory(
            self.layers[start:end], total=opts.device_total(worker), optimizer=opts.optimizer,
            num_microbatches=opts.num_microbatches, is_last=last, stage_index=index, num_stages=len(order),
            schedule=opts.schedule, max_inflight=opts.max_inflight, backend=worker.backend,
            activation_safety=opts.activation_safety, available=worker.memory_available, engine=opts.engine,
            param_dtype_bytes=opts.param_dtype_bytes, offload=opts.offload, offload_ring=opts.offload_ring,
            **opts.memory_kwargs(worker.backend))
        return StagePlan(index, worker.worker_id, worker.name, worker.backend, start, end, memory,
                         compute_s=compute_time(self.flops_before[end] - self.flops_before[start],
                                                worker.measured_flops),
                         comm_s=sum(d["total_s"] for d in detail.values()),
                         boundary_bytes=0 if last else self.layers[end - 1].activation_bytes,
                         overlap=opts.async_transport, comm_detail=detail)


def eligible_workers(workers: list[WorkerProfile], opts: PlannerOptions):
    """(workers the plan may use, {excluded worker name: reason})."""
    usable, excluded = [], {}
    for w in workers:
        have = set(w.supported_ops.get(opts.dtype, ())) if w.supported_ops is not None else None
        missing = sorted(set(opts.required_ops) - have) if have is not None else []
        budget, _ = usable_bytes(opts.device_total(w), w.backend, available=w.memory_available,
                                 **opts.memory_kwargs(w.backend))
        reason = (f"backend {w.backend} not allowed" if w.backend not in opts.allow_backends else
                  f"no {opts.dtype} support" if opts.dtype not in w.supported_dtypes else
                  f"cannot run {', '.join(missing)} in {opts.dtype}" if missing else
                  "memory below safety margin" if budget <= 0 else None)
        if reason is None:
            usable.append(w)
        else:
            excluded[w.name] = reason
    return usable, excluded


def _assemble(strategy: str, order, bounds, coster: StageCoster, excluded: dict) -> Plan:
    plan = Plan(strategy, [coster(order, i, a, b) for i, (a, b) in enumerate(bounds)],
                coster.opts.num_microbatches, excluded=dict(excluded))
    widths = [b - a for a, b in bounds]
    if sum(widths) != len(coster.layers) or min(widths, default=0) <= 0:
        plan.violations.append("partition does not cover every layer exactly once")
    plan.violations += [f"stage {s.stage_index} on {s.worker_name} needs {s.memory.required / GB:.2f} GB but only "
                        f"{s.memory.budget / GB:.2f} GB is usable" for s in plan.stages if not s.memory.fits]
    return plan


def even_bounds(n_layers: int, k: int) -> list[tuple[int, int]]:
    return [(n_layers * i // k, n_layers * (i + 1) // k) for i in range(k)]


def split_by_weights(n_layers: int, weights: list[float], layer_cost: list[float]) -> list[tuple[int, int]]:
    """Contiguous ranges whose cumulative cost follows the cumulative weight share.

    Cut i goes to the layer boundary whose cumulative cost is nearest the
    target share, kept far enough from its neighbours that every range has at
    least one layer.
    """
    k = len(weights)
    costs = layer_cost if sum(layer_cost) > 0 else [1.0] * n_layers
    before = list(itertools.accumulate(costs, initial=0.0))
    targets = [s * before[-1] for s in itertools.accumulate(w / sum(weights) for w in weights)]
    cuts, prev = [], 0
    for i in range(k - 1):
        lo, hi = prev + 1, n_layers - (k - 1 - i)
        cut = min(range(lo, hi + 1), key=lambda b: (abs(before[b] - targets[i]), b))
        cuts.append(cut)
        prev = cut
    edges = [0] + cuts + [n_layers]
    return list(zip(edges, edges[1:]))


def _preferred(a, b, tol: float) -> bool:
    """Is candidate a = (bottleneck, boundary bytes) better than b?  Faster wins; near-ties go to fewer bytes."""
    if b is None or b[0] == math.inf:
        return a[0] < math.inf
    if a[0] < b[0] * (1 - tol):
        return True
    return a[0] <= b[0] * (1 + tol) and a[1] < b[1]


def minimax_bounds(coster: StageCoster, order: list[WorkerProfile]):
    """Cut positions minimising the slowest stage for a fixed worker order, or None if nothing fits."""
    n, k, tol = len(coster.layers), len(order), coster.opts.tie_tolerance

    @lru_cache(maxsize=None)
    def best(stage: int, start: int):
        """(bottleneck, bytes, cuts) for stages stage..k-1 covering layers start..n-1."""
        if stage == k - 1:
            s = coster(order, stage, start, n)
            return (s.time_per_mb, s.boundary_bytes, (n,)) if s.memory.fits else None
        chosen = None
        for end in range(start + 1, n - (k - 1 - stage) + 1):
            s = coster(order, stage, start, end)
            if not s.memory.fits:
                continue
            rest = best(stage + 1, end)
            if rest is None:
                continue
            cand = (max(s.time_per_mb, rest[0]), s.boundary_bytes + rest[1], (end,) + rest[2])
            if _preferred(cand, chosen, tol):
                chosen = cand
        return chosen

    found = best(0, 0)
    if found is None:
        return None
    edges = (0,) + found[2]
    return found[:2], list(zip(edges, edges[1:]))


def _distinct_orderings(ws: list[WorkerProfile], k: int, network: NetworkModel):
    """Ordered k-subsets of ``ws``, once per arrangement of distinguishable workers."""
    ids = [w.worker_id for w in ws]

    def fingerprint(w: WorkerProfile) -> tuple:
        links = sorted((network.latency.get((w.worker_id, o)), network.bandwidth.get((w.worker_id, o)),
                        (w.worker_id, o) in network.device_links) for o in ids if o != w.worker_id)
        return (w.backend, w.memory_total, w.measured_flops, w.host, w.d2h_Bps, w.h2d_Bps, w.memory_available,
                w.unified_memory, tuple(links))

    prints = {w.worker_id: fingerprint(w) for w in ws}
    seen = set()
    for order in itertools.permutations(ws, k):
        sig = tuple(prints[w.worker_id] for w in order)
        if sig not in seen:
            seen.add(sig)
            yield list(order)


def plan_equal(layers, workers, network, opts) -> Plan:
    ws, excluded = eligible_workers(workers, opts)
    k = min(opts.num_stages or len(ws), len(ws), len(layers))
    return _assemble("equal", ws[:k], even_bounds(len(layers), k), StageCoster(layers, network, opts), excluded)


def plan_compute(layers, workers, network, opts) -> Plan:
    ws, excluded = eligible_workers(workers, opts)
    k = min(opts.num_stages or len(ws), len(ws), len(layers))
    fastest = set(id(w) for w in sorted(ws, key=lambda w: -w.measured_flops)[:k])
    order = [w for w in ws if id(w) in fastest]  # the user's order among the chosen workers
    bounds = split_by_weights(len(layers), [w.measured_flops for w in order], [max(l.flops, 1.0) for l in layers])
    return _assemble("compute", order, bounds, StageCoster(layers, network, opts), excluded)


def plan_auto(layers, workers, network, opts) -> Plan:
    ws, excluded = eligible_workers(workers, opts)
    coster = StageCoster(layers, network, opts)
    counts = [opts.num_stages] if opts.num_stages else range(1, min(len(ws), len(layers)) + 1)
    winner = None  # ((bottleneck, bytes), order, bounds)
    budget = opts.max_orderings
    for k in counts:
        for order in _distinct_orderings(ws, k, network):
            budget -= 1
            if budget < 0:
                break
            found = minimax_bounds(coster, order)
            if found is None:
                continue
            (t, nbytes), bounds = found
            if winner is None:
                winner = ((t, nbytes), order, bounds)
                continue
            (bt, bbytes), border, _ = winner
            near = abs(t - bt) <= bt * 0.02
            if t < bt * 0.98 or (near and (k, nbytes) < (len(border), bbytes)):
                winner = ((t, nbytes), order, bounds)
    if winner is None:
        plan = Plan("auto", [], opts.num_microbatches, excluded=excluded)
        plan.violations.append("no contiguous partition fits the memory budgets of the eligible workers")
        return plan
    return _assemble("auto", winner[1], winner[2], coster, excluded)


def plan_manual(layers, workers, network, opts, assignments: list[tuple[str, int, int]]) -> Plan:
    lookup = {w.name: w for w in workers}
    lookup.update({w.worker_id: w for w in workers})
    unknown = [wid for wid, _a, _b in assignments if wid not in lookup]
    if unknown:
        raise ValueError(f"manual placement names unknown worker {unknown[0]!r}")
    order = [lookup[wid] for wid, _a, _b in assignments]
    return _assemble("manual", order, [(a, b) for _, a, b in assignments], StageCoster(layers, network, opts), {})


STRATEGIES = {"equal": plan_equal, "compute": plan_compute, "auto": plan_auto, "topology_aware": plan_auto}


def make_plan(strategy: str, layers, workers, network: NetworkModel | None = None,
              opts: PlannerOptions | None = None) -> Plan:
    planner = STRATEGIES.get(strategy)
    if planner is None:
        raise ValueError(f"unknown strategy {strategy!r}")
    return planner(layers, workers, network or NetworkModel(), opts or PlannerOptions())


def b200_box(num_gpus: int = 8, memory_gb: float = 180.0, tflops: float = 1.2e15, host: str = "b200-box"):
    """Worker profiles and network model of one NVSwitch box of B200s (NCCL link between every pair)."""
    ws = [WorkerProfile(f"{host}:gpu{i}", f"gpu{i}", "cuda", int(memory_gb * GB), tflops, host=host,
                        d2h_Bps=55e9, h2d_Bps=55e9) for i in range(num_gpus)]
    network = NetworkModel(device_links={(a.worker_id, b.worker_id) for a in ws for b in ws if a is not b})
    return ws, network

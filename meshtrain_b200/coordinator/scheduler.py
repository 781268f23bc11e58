"""Registered workers + a job config -> a placement plan (reference coordinator/scheduler.py:17-97).

The coordinator never builds weights: the model is profiled analytically (GPT /
Llama) or on the ``meta`` device, then the planner runs.  GPU workers on the
same box are joined by NVLink device links when the job moves tensors with
NCCL (``network.tensor_transport: nccl``), otherwise every boundary is a host
hop (D2H -> TCP -> H2D) priced from the measured link matrix.
"""

from __future__ import annotations

import dataclasses
import itertools

from meshtrain_b200.config import MeshTrainConfig
from meshtrain_b200.coordinator.state import WorkerRecord
from meshtrain_b200.parallel.placement import config_mode
from meshtrain_b200.planner.cost import NetworkModel
from meshtrain_b200.planner.graph import profiles_for
from meshtrain_b200.planner.partition import Plan, PlannerOptions, WorkerProfile, make_plan, plan_manual

# FLOP/s assumed for a worker that has not been benchmarked (conservative).
UNBENCHMARKED_FLOPS = {"cuda": 5e12, "mps": 1e12, "cpu": 5e10}
_DTYPE_CAPS = (("float32", "supports_fp32"), ("float16", "supports_fp16"), ("bfloat16", "supports_bf16"),
               ("float64", "supports_fp64"))


def live_cuda_budget(total: int, memory: dict) -> int | None:
    """Bytes an idle CUDA worker can still hand to a new stage.

    Free memory plus the allocator's idle cache, never more than total minus
    live allocations; cached bytes beyond the device's capacity (oversubscribed
    pools) do not count.
    """
    if memory.get("free") is None:
        return None
    allocated = max(0, int(memory.get("allocated", 0)))
    reserved = max(0, int(memory.get("reserved", 0)))
    cache = max(0, reserved - allocated) if reserved <= total else 0
    return min(max(0, total - allocated), max(0, int(memory["free"]) + cache))


def worker_profile(w: WorkerRecord) -> WorkerProfile:
    dev = w.device_info or {}
    available = None
    if w.backend == "cpu":
        total = int(w.hardware.get("ram_available") or w.hardware.get("ram_total", 0))
    else:
        total = int(dev.get("memory_total", 0))
        if w.backend == "cuda":
            available = live_cuda_budget(total, w.memory or {})
    caps = w.capabilities or {}
    supported_ops = None
    if caps.get("dtypes") is not None:  # this package's probe report: {"dtypes": [...], "ops": {op: [dtypes]}}
        dtypes = tuple(caps["dtypes"])
        supported_ops = {}
        for op, dts in (caps.get("ops") or {}).items():
            for dt in dts:
                supported_ops.setdefault(dt, []).append(op)
    elif caps:  # reference-style report
        dtypes = tuple(dt for dt, key in _DTYPE_CAPS if caps.get(key))
        supported_ops = caps.get("op_capabilities")
    else:
        dtypes = ("float32", "float16", "bfloat16") if w.backend == "mps" else \
            ("float32", "float16", "bfloat16", "float64")
    bench = w.benchmark or {}
    flops = bench.get("measured_flops") or UNBENCHMARKED_FLOPS.get(w.backend, 5e10)
    copy = 0.0 if w.backend == "cpu" else 6e9  # unmeasured accelerator: ~PCIe 3 x8
    return WorkerProfile(w.worker_id, w.name, w.backend, total, float(flops),
                         unified_memory=bool(dev.get("unified_memory")), supported_dtypes=dtypes,
                         supported_ops=supported_ops, d2h_Bps=float(bench.get("d2h_Bps", copy)),
                         h2d_Bps=float(bench.get("h2d_Bps", copy)), memory_available=available, host=w.host_key)


def add_device_links(network: NetworkModel, workers: list[WorkerRecord]) -> NetworkModel:
    """Mark every ordered pair of CUDA workers on one box as an NVLink (NCCL) link."""
    for a, b in itertools.permutations(workers, 2):
        if a.backend == b.backend == "cuda" and a.host_key == b.host_key:
            network.device_links.add((a.worker_id, b.worker_id))
    return network


def _model_profiles(cfg: MeshTrainConfig):
    spec = cfg.build_model_spec()
    mb = cfg.training.microbatch_size or cfg.training.batch_size
    return spec, profiles_for(spec, mb)


def recompute_units(cfg: MeshTrainConfig, layers=None) -> set[int]:
    """Units a device-engine job recomputes in backward (``training.activation_recompute``)."""
    if cfg.network.tensor_transport != "nccl" or cfg.training.activation_recompute == "none":
        return set()
    from meshtrain_b200.parallel.recompute import choose_units

    return choose_units(cfg.training.activation_recompute, layers if layers is not None else _model_profiles(cfg)[1])


def layer_profiles(cfg: MeshTrainConfig):
    """Per-unit profiles of the job's model; device-engine jobs see their recomputed units as such."""
    from meshtrain_b200.parallel.recompute import apply_to_profiles

    spec, layers = _model_profiles(cfg)
    units = recompute_units(cfg, layers)
    return spec, apply_to_profiles(layers, units) if units else layers


def plan_job(cfg: MeshTrainConfig, workers: list[WorkerRecord], network: NetworkModel | None = None,
             budget_overrides: dict[str, int] | None = None) -> Plan:
    spec, layers = layer_profiles(cfg)
    profiles = [worker_profile(w) for w in workers]
    if cfg.workers.require:
        known = {p.worker_id for p in profiles} | {p.name for p in profiles}
        missing = set(cfg.workers.require) - known
        if missing:
            raise ValueError(f"required workers not online: {sorted(missing)}")
    network = network or NetworkModel()
    device_engine = cfg.network.tensor_transport == "nccl"
    if device_engine:
        add_device_links(network, workers)
    pc = cfg.placement
    legacy_margin = pc.memory_headroom_fraction is not None or pc.memory_headroom_min_gb is not None
    import torch

    opts = PlannerOptions(
        optimizer=cfg.training.optimizer, num_microbatches=cfg.training.num_microbatches,
        allow_backends=tuple(cfg.workers.allow), dtype=cfg.model.dtype,
        headroom_fraction=(pc.memory_headroom_fraction or 0.0) if legacy_margin else None,
        headroom_min_bytes=int((pc.memory_headroom_min_gb or 0.0) * 1024 ** 3) if legacy_margin else None,
        activation_safety=pc.activation_overhead_factor, num_stages=pc.num_stages, schedule=cfg.pipeline.schedule,
        max_inflight=cfg.pipeline.max_inflight_microbatches, safety_factors=cfg.memory.safety_factors(),
        framework_reserve=cfg.memory.framework_reserve_bytes(), budget_overrides=dict(budget_overrides or {}),
        async_transport=cfg.transport.async_,
        required_ops=tuple(getattr(spec, "required_ops", ())) + (
            ("adamw",) if cfg.training.optimizer in ("adam", "adamw") else ()),
        engine="device" if device_engine else "autograd",
        param_dtype_bytes=torch.empty((), dtype=getattr(torch, cfg.model.dtype)).element_size(),
        offload=config_mode(cfg.offload) == "host",
        offload_ring=dict(chunk_mb=cfg.offload.chunk_mb, prefetch_ahead=cfg.offload.prefetch_ahead,
                          device_budget_gb=cfg.offload.device_budget_gb),
    )

    def place(options):
        if pc.strategy == "manual":
            return plan_manual(layers, profiles, network, options,
                               [(s.worker or s.device, s.layers[0], s.layers[1]) for s in pc.stages])
        return make_plan(pc.strategy, layers, profiles, network, options)

    plan = place(opts)
    plan.state_offload = opts.offload
    if device_engine and config_mode(cfg.offload) == "auto" and not plan.feasible:
        # the optimizer state's tier is "auto": move it to host memory when the resident plan does not fit
        offloaded = place(dataclasses.replace(opts, offload=True))
        if offloaded.feasible or not plan.stages:
            plan = offloaded
            plan.state_offload = True
    return plan


def interleaved_layout(cfg: MeshTrainConfig, plan: Plan) -> list[dict] | None:
    """Model chunks and memory estimate of each stage of a device-engine job with
    ``pipeline.virtual_stages`` v > 1 (interleaved 1F1B), or None for a plain layout.

    The plan fixes the workers and their order (rank i runs the plan's stage i); the
    model is then cut into v x S FLOP-balanced pieces (``interleaved_split``) and rank i
    holds pieces i, i + S, ...  Each rank's estimate counts the chunk-forwards its
    interleaved program keeps alive against that worker's memory.
    """
    v, S = cfg.pipeline.virtual_stages, len(plan.stages)
    if v <= 1 or S <= 1 or cfg.network.tensor_transport != "nccl":
        return None
    M = cfg.training.num_microbatches
    if M % S:
        raise ValueError(f"pipeline.virtual_stages {v} needs the number of microbatches ({M}) to be a multiple "
                         f"of the number of stages ({S})")
    from meshtrain_b200.parallel.engine import interleaved_split
    from meshtrain_b200.planner.memory import estimate_interleaved_rank
    import torch

    spec, layers = layer_profiles(cfg)
    if v * S > len(layers):
        raise ValueError(f"{v} x {S} virtual stages need at least that many partition units ({len(layers)})")
    pieces = interleaved_split([max(lay.flops, 1.0) for lay in layers], S, v)
    eb = torch.empty((), dtype=getattr(torch, cfg.model.dtype)).element_size()
    offload = getattr(plan, "state_offload", config_mode(cfg.offload) == "host")
    out = []
    for rank, stage in enumerate(plan.stages):
        est = estimate_interleaved_rank(
            layers, pieces, rank, S, v, M, total=stage.memory.total, optimizer=cfg.training.optimizer,
            param_dtype_bytes=eb, offload=offload,
            offload_ring=dict(chunk_mb=cfg.offload.chunk_mb, prefetch_ahead=cfg.offload.prefetch_ahead,
                              device_budget_gb=cfg.offload.device_budget_gb),
            safety_factor=cfg.memory.safety_factors().get(stage.backend, cfg.memory.safety_factor),
            framework_reserve=cfg.memory.framework_reserve_bytes().get(stage.backend, 0))
        out.append({"chunk_ranges": [list(pieces[c * S + rank]) for c in range(v)], "memory": est})
    return out

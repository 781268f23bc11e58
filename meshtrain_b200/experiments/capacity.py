"""Capacity: the largest model trainable on each device alone vs. on the mesh.

Same question and the same two ratios as the reference's experiment
(experiments/capacity.py:1-243):

    capacity_gain      = P_mesh_max / max_i P_single_max[i]
    throughput_penalty = steps/s(best single device, its largest model) / steps/s(mesh, its largest model)

Each *target* (one device alone, or the whole mesh) climbs a ladder of model
sizes until the first size it cannot hold; the last size it held is its limit.

Modes:

* ``emulated`` - a heterogeneous cluster scaled down ``SCALE`` times and emulated
  by CPU processes. A target holds a size when the planner finds a placement
  within the emulated budgets; the two limits that decide the ratios are then
  trained for real, and the bytes each stage held are reported against its budget.
* ``b200`` - planner-only: largest Llama-style size per number of B200s (180 GB,
  NVLink), with fp32 master weights + Adam moments on the device or in host DRAM.
* ``hardware`` - every rung is submitted to the running cluster as a job, first
  pinned to each worker alone, then planned across the mesh; a failed job (out of
  memory, refused plan) ends that target's climb.
"""

from __future__ import annotations

import statistics
import time
from dataclasses import dataclass, field

from meshtrain_b200.experiments.emulation import MB, EmulatedWorker, profile_emulated
from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.planner.cost import NetworkModel
from meshtrain_b200.planner.graph import profile_model
from meshtrain_b200.planner.partition import PlannerOptions, make_plan

GB = 1024 ** 3
SCALE = 32
# (name, real device memory) of the cluster being emulated
TARGET = [("gpu-8g", 8 * GB), ("gpu-12g", 12 * GB), ("laptop-16g", int(16 * GB * 2 / 3))]
BATCH, MICRO = 8, 2
# (blocks, hidden) rungs, smallest first
SIZES = [(2, 128), (4, 192), (4, 256), (6, 256), (6, 320), (6, 384), (8, 384), (8, 448), (8, 512), (10, 512),
         (12, 512), (12, 576), (14, 576), (14, 640), (16, 640), (16, 704), (18, 704), (20, 768)]
MESH = "mesh"


def model_cfg(blocks: int, hidden: int) -> dict:
    """Config of one rung: the tiny-transformer family at a given depth and width."""
    return dict(type="tiny_transformer", layers=blocks, hidden_size=hidden, heads=8, vocab_size=1024, seq_len=64)


@dataclass
class Rung:
    blocks: int
    hidden: int

    @property
    def cfg(self) -> dict:
        return model_cfg(self.blocks, self.hidden)

    @property
    def label(self) -> str:
        return f"{self.blocks}x{self.hidden}"


@dataclass
class Climb:
    """Progress of one target up the ladder."""

    name: str
    limit: tuple | None = None  # (params, rung, plan-or-job info) of the largest size held so far
    stopped_by: str | None = None
    per_rung: dict = field(default_factory=dict)  # rung label -> cell text

    @property
    def climbing(self) -> bool:
        return self.stopped_by is None

    def held(self, params: int, rung: Rung, info, cell: str = "fits") -> None:
        self.limit = (params, rung, info)
        self.per_rung[rung.label] = cell

    def failed(self, rung: Rung, why: str) -> None:
        self.stopped_by = why or "failed"
        self.per_rung[rung.label] = "-"


def _planner_options(stages: int | None) -> PlannerOptions:
    return PlannerOptions(optimizer="adamw", num_microbatches=BATCH // MICRO, headroom_fraction=0.10,
                          headroom_min_bytes=8 * MB, num_stages=stages)


def _train_plan(cfg: dict, plan, threads: dict[str, int], steps: int) -> dict:
    """Train ``cfg`` on the plan's stages as CPU processes; throughput, losses and bytes held per stage."""
    settings = PipelineSettings("capacity", steps=steps, batch_size=BATCH, num_microbatches=BATCH // MICRO,
                                log_every=10 ** 6, timeout_s=300)
    stages = [LocalStage((st.start, st.end), "cpu", threads=threads[st.worker_id]) for st in plan.stages]
    results = run_local_pipeline(cfg, stages, settings, optimizer="adamw", lr=3e-4, timeout_s=3600)
    first = results[0]
    timed = first.step_metrics[1:] or first.step_metrics  # the first step also builds the optimizer state
    holdings = []
    for st, res in zip(plan.stages, results):
        last = res.step_metrics[-1]["memory"]
        activations = max(rec["memory"]["saved_activations_peak"] for rec in res.step_metrics)
        resident = last["parameters"] + last["gradients"] + last["optimizer_state"]
        holdings.append((st.worker_name, resident + activations, st.memory.budget))
    return {"steps_per_s": 1.0 / statistics.median(r["step_s"] for r in timed), "held": holdings,
            "losses": (first.losses[0], first.losses[-1])}


def _holdings_text(run: dict) -> str:
    return ", ".join(f"{who}: {used / MB:.0f}/{budget / MB:.0f} MB" for who, used, budget in run["held"])


def run_emulated(steps: int = 5, write_doc: bool = True, sizes=SIZES) -> str:
    workers = [EmulatedWorker(name, threads=1, memory_budget_bytes=mem // SCALE, label=f"{mem / GB:.1f} GB / {SCALE}")
               for name, mem in TARGET]
    profiles = profile_emulated(workers)
    climbs = {p.name: Climb(p.name) for p in profiles}
    climbs[MESH] = Climb(MESH)
    rows = []
    for rung in (Rung(b, h) for b, h in sizes):
        if not any(c.climbing for c in climbs.values()):
            break
        spec = build_model_spec(rung.cfg)
        params = spec.parameter_count()
        layers = profile_model(spec, MICRO)
        for prof in profiles:
            if climbs[prof.name].climbing:
                plan = make_plan("auto", layers, [prof], NetworkModel(), _planner_options(1))
                if plan.feasible:
                    climbs[prof.name].held(params, rung, plan)
                else:
                    climbs[prof.name].failed(rung, "; ".join(plan.violations))
        total_required = "-"
        if climbs[MESH].climbing:
            plan = make_plan("auto", layers, profiles, NetworkModel(), _planner_options(None))
            if plan.stages:
                total_required = f"{sum(st.memory.required for st in plan.stages) / MB:.0f} MB"
            if plan.feasible:
                climbs[MESH].held(params, rung, plan, f"fits ({len(plan.stages)} stages)")
            else:
                climbs[MESH].failed(rung, "; ".join(plan.violations))
        rows.append([rung.label, f"{params / 1e6:.1f}M",
                     *[climbs[p.name].per_rung.get(rung.label, "-") for p in profiles],
                     climbs[MESH].per_rung.get(rung.label, "-"), total_required])

    singles = [c for name, c in climbs.items() if name != MESH and c.limit]
    if not singles or climbs[MESH].limit is None:
        raise RuntimeError("no tested size fits a single device or the mesh")
    best = max(singles, key=lambda c: c.limit[0])
    p_single, rung_single, plan_single = best.limit
    p_mesh, rung_mesh, plan_mesh = climbs[MESH].limit
    threads = {w.name: w.threads for w in workers}
    alone = _train_plan(rung_single.cfg, plan_single, threads, steps)
    mesh = _train_plan(rung_mesh.cfg, plan_mesh, threads, steps)
    gain = p_mesh / p_single
    penalty = alone["steps_per_s"] / mesh["steps_per_s"]

    def result_row(kind, params, where, run):
        first, last = run["losses"]
        return [kind, f"{params / 1e6:.1f}M", where, f"{run['steps_per_s']:.3f}", _holdings_text(run),
                f"{first:.3f} -> {last:.3f}"]

    md = "\n\n".join([
        environment_line(),
        f"**Mode: emulated.** Cluster memory scaled down {SCALE}x and emulated by single-threaded CPU processes; "
        "limits are the planner's accounting (params + grads + AdamW state + saved activations + temporaries, "
        f"10% headroom), not real out-of-memory errors. Tiny transformer family, AdamW, batch {BATCH}.",
        md_table(["worker", "real memory", "emulated budget", "measured GFLOP/s"],
                 [[w.name, f"{mem / GB:.1f} GB", f"{w.memory_budget_bytes / MB:.0f} MB",
                   f"{p.measured_flops / 1e9:.1f}"] for (_, mem), w, p in zip(TARGET, workers, profiles)]),
        md_table(["model", "params", *[f"{w.name} alone" for w in workers], "mesh", "mesh total required"], rows),
        md_table(["", "P_max", "device(s)", "steps/s", "MB held/budget", "loss"],
                 [result_row("single device", p_single, best.name, alone),
                  result_row("mesh", p_mesh, " -> ".join(st.worker_name for st in plan_mesh.stages), mesh)]),
        f"**capacity_gain = {p_mesh / 1e6:.1f}M / {p_single / 1e6:.1f}M = {gain:.2f}x**; throughput penalty "
        f"{penalty:.2f}x (emulated: one core per worker, loopback links - only the capacity ratio is meaningful)."])
    if write_doc:
        update_section("capacity-emulated", md)
    return md


def _llama_cfg(blocks: int) -> dict:
    return dict(type="llama", layers=blocks, hidden_size=4096, heads=32, n_kv_heads=8, ffn_hidden=14336,
                vocab_size=128256, seq_len=4096, dtype="bfloat16")


def largest_llama(gpus: int, offload: bool, max_blocks: int = 160) -> tuple[int, int] | None:
    """(blocks, parameters) of the largest Llama-style model the device planner places on ``gpus`` B200s.

    The planner's verdict is monotone in depth, so a bisection over the block count
    (multiples of four) finds the boundary with a handful of plans.
    """
    from meshtrain_b200.api import plan_device_pipeline

    def fits(units: int) -> bool:  # units of four blocks
        try:
            plan_device_pipeline(build_model_spec(_llama_cfg(4 * units)), gpus, 32, 1, "1f1b", "adam",
                                 offload=offload, memory_gb=180.0)
        except RuntimeError:
            return False
        return True

    # the shallowest model with at least one partition unit per GPU
    lo, hi = 1, max_blocks // 4
    while lo <= hi and build_model_spec(_llama_cfg(4 * lo)).num_layers < gpus:
        lo += 1
    if lo > hi or not fits(lo):
        return None
    while lo < hi:  # invariant: lo fits
        mid = (lo + hi + 1) // 2
        if fits(mid):
            lo = mid
        else:
            hi = mid - 1
    blocks = 4 * lo
    return blocks, build_model_spec(_llama_cfg(blocks)).parameter_count()


def b200_capacity(write_doc: bool = True) -> str:
    """Largest Llama-family model (d=4096 blocks, seq 4096) per number of B200s, planner-only."""
    rows = []
    for gpus in (1, 2, 4, 8):
        for offload in (False, True):
            found = largest_llama(gpus, offload)
            rows.append([gpus, "host" if offload else "device", f"{found[0]} blocks" if found else "-",
                         f"{found[1] / 1e9:.1f} B" if found else "-"])
    md = "\n\n".join([environment_line(), "Planner-only: largest Llama-style model (d 4096, GQA 32/8, SwiGLU 14336, "
                      "seq 4096, 32 microbatches of 1, Adam, bf16 compute + fp32 master) that fits N B200s "
                      "(180 GB each) with fp32 master weights + Adam moments on the device or offloaded to host DRAM.",
                      md_table(["B200s", "optimizer state", "largest model", "parameters"], rows)])
    if write_doc:
        update_section("capacity-b200", md)
    return md


class _JobRunner:
    """Submits one capacity trial to the coordinator and waits for its outcome."""

    def __init__(self, client, steps: int, mesh_size: int, poll_s: float):
        self.client, self.steps, self.mesh_size, self.poll_s = client, steps, mesh_size, poll_s

    def config(self, rung: Rung, worker: str | None) -> dict:
        cfg = {"job": {"name": "capacity"}, "model": rung.cfg, "network": {"timeout_s": 300},
               "training": dict(batch_size=BATCH, microbatch_size=MICRO, learning_rate=3e-4, optimizer="adamw",
                                steps=self.steps, log_every=1)}
        if worker is None:
            cfg["placement"] = dict(strategy="auto", num_stages=self.mesh_size, enforce_memory_check=True)
        else:  # the whole model pinned to one worker; its own memory decides
            layers = build_model_spec(rung.cfg).num_layers
            cfg["placement"] = dict(strategy="manual", enforce_memory_check=False,
                                    stages=[{"worker": worker, "layers": [0, layers]}])
        return cfg

    def run(self, rung: Rung, worker: str | None) -> dict:
        try:
            job_id = self.client.start_job(self.config(rung, worker))["job_id"]
        except Exception as exc:  # noqa: BLE001 - a refused plan is a size that does not fit
            return {"ok": False, "error": str(exc)[:200]}
        job = self.client.job(job_id)
        while job["status"] == "RUNNING":
            time.sleep(self.poll_s)
            job = self.client.job(job_id)
        mean = (job.get("summary") or {}).get("mean_step_s")
        ok = job["status"] == "COMPLETED"
        return {"ok": ok, "error": job.get("error"), "stages": len(job["stage_workers"]),
                "steps_per_s": 1.0 / mean if ok and mean else None}


def run_hardware(client, sizes=SIZES, steps: int = 5, write_doc: bool = True, poll_s: float = 1.0) -> str:
    online = [w["worker_id"] for w in client.status()["workers"] if w["status"] == "ONLINE"]
    if len(online) < 2:
        raise ValueError("the hardware capacity comparison needs at least two online workers")
    runner = _JobRunner(client, steps, len(online), poll_s)
    climbs = {wid: Climb(wid) for wid in online}
    climbs[MESH] = Climb(MESH)
    for rung in (Rung(b, h) for b, h in sizes):
        active = [c for c in climbs.values() if c.climbing]
        if not active:
            break
        params = build_model_spec(rung.cfg).parameter_count()
        for climb in active:  # each worker alone first, the mesh last
            out = runner.run(rung, None if climb.name == MESH else climb.name)
            if out["ok"]:
                climb.held(params, rung, out)
            else:
                climb.failed(rung, out["error"])

    def clean(text):
        return (text or "").replace("\n", " ").replace("|", "/")[:120]

    def row(climb: Climb):
        params, _, out = climb.limit or (0, None, {})
        stages = (out.get("stages", "-") if climb.name == MESH else 1) if climb.limit else "-"
        return [climb.name, f"{params / 1e6:.1f}M", f"{out.get('steps_per_s') or 0:.3f}", stages,
                clean(climb.stopped_by)]

    table = [row(climbs[w]) for w in online] + [row(climbs[MESH])]
    parts = [environment_line(), f"**Mode: hardware** (real devices through the coordinator); mesh trials use all "
             f"{len(online)} online workers. P_max is the largest size that trained.",
             md_table(["device", "P_max", "steps/s at P_max", "stages", "first failure"], table)]
    held_alone = [climbs[w].limit for w in online if climbs[w].limit]
    if held_alone and climbs[MESH].limit:
        p_best, _, out_best = max(held_alone, key=lambda lim: lim[0])
        p_mesh, _, out_mesh = climbs[MESH].limit
        parts.append(f"capacity_gain = {p_mesh / p_best:.2f}x, throughput penalty = "
                     f"{(out_best['steps_per_s'] or 0) / (out_mesh['steps_per_s'] or 1):.2f}x")
    md = "\n\n".join(parts)
    if write_doc:
        update_section("capacity-hardware", md)
    return md


def run_experiment5(mode: str = "emulated", cluster_file: str | None = None, steps: int = 5, *, client=None) -> str:
    """Dispatch of ``meshtrain experiment capacity --mode emulated|b200|hardware``."""
    runners = {"emulated": lambda: run_emulated(steps=steps), "b200": b200_capacity}
    if mode in runners:
        return runners[mode]()
    if client is None:
        from meshtrain_b200.cli import client_from

        client = client_from()
    try:
        return run_hardware(client, steps=steps)
    finally:
        client.close()

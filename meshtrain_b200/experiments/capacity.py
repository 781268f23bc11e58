"""Capacity: the largest model trainable on each device alone vs. on the mesh (reference
experiments/capacity.py:1-243).

    capacity_gain      = P_mesh_max / max_i P_single_max[i]
    throughput_penalty = steps/s(best single device, its largest model) / steps/s(mesh, its largest model)

Modes:

* ``emulated`` - a heterogeneous cluster scaled down ``SCALE`` times and emulated
  by CPU processes; feasibility from the planner's accounting against the
  emulated budgets, then the largest models really train and the bytes each
  stage held are checked against its budget;
* ``b200`` - planner-only: largest GPT/Llama size per number of B200s (180 GB,
  NVLink), with and without host offload of master weights + Adam state;
* ``hardware`` - every size is submitted to the running cluster, first to each
  worker alone, then to the whole mesh; a failure (out of memory) marks the limit.
"""

from __future__ import annotations

import statistics
import time

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
TARGET = [("gpu-8g", 8 * GB), ("gpu-12g", 12 * GB), ("laptop-16g", int(16 * GB * 2 / 3))]
BATCH, MICRO = 8, 2
SIZES = [(2, 128), (4, 192), (4, 256), (6, 256), (6, 320), (6, 384), (8, 384), (8, 448), (8, 512), (10, 512),
         (12, 512), (12, 576), (14, 576), (14, 640), (16, 640), (16, 704), (18, 704), (20, 768)]


def model_cfg(blocks: int, hidden: int) -> dict:
    return {"type": "tiny_transformer", "layers": blocks, "hidden_size": hidden, "heads": 8, "vocab_size": 1024,
            "seq_len": 64}


def _opts(num_stages=None) -> PlannerOptions:
    return PlannerOptions(optimizer="adamw", num_microbatches=BATCH // MICRO, headroom_fraction=0.10,
                          headroom_min_bytes=8 * MB, num_stages=num_stages)


def _train(cfg: dict, plan, threads: dict[str, int], steps: int) -> dict:
    stages = [LocalStage((s.start, s.end), "cpu", threads=threads[s.worker_id]) for s in plan.stages]
    settings = PipelineSettings("capacity", steps=steps, batch_size=BATCH, num_microbatches=BATCH // MICRO,
                                log_every=10 ** 6, timeout_s=300)
    res = run_local_pipeline(cfg, stages, settings, optimizer="adamw", lr=3e-4, timeout_s=3600)
    step_s = statistics.median(m["step_s"] for m in res[0].step_metrics[1:] or res[0].step_metrics)
    held = []
    for r, s in zip(res, plan.stages):
        m = r.step_metrics[-1]["memory"]  # optimizer state exists after the first update
        peak = max(x["memory"]["saved_activations_peak"] for x in r.step_metrics)
        held.append((s.worker_name, m["parameters"] + m["gradients"] + m["optimizer_state"] + peak, s.memory.budget))
    return {"steps_per_s": 1 / step_s, "held": held, "loss_first": res[0].losses[0], "loss_last": res[0].losses[-1]}


def run_emulated(steps: int = 5, write_doc: bool = True, sizes=SIZES) -> str:
    workers = [EmulatedWorker(n, threads=1, memory_budget_bytes=mem // SCALE, label=f"{mem / GB:.1f} GB / {SCALE}")
               for n, mem in TARGET]
    profiles = profile_emulated(workers)
    threads = {w.name: w.threads for w in workers}
    rows, single_max, mesh_max = [], {}, None
    for blocks, hidden in sizes:
        cfg = model_cfg(blocks, hidden)
        spec = build_model_spec(cfg)
        layers = profile_model(spec, MICRO)
        P = spec.parameter_count()
        cells = []
        for p in profiles:
            plan = make_plan("auto", layers, [p], NetworkModel(), _opts(num_stages=1))
            cells.append("fits" if plan.feasible else "-")
            if plan.feasible:
                single_max[p.name] = (P, cfg, plan)
        mesh = make_plan("auto", layers, profiles, NetworkModel(), _opts())
        if mesh.feasible:
            mesh_max = (P, cfg, mesh)
        need = sum(s.memory.required for s in mesh.stages) if mesh.stages else None
        rows.append([f"{blocks}x{hidden}", f"{P / 1e6:.1f}M", *cells,
                     f"fits ({len(mesh.stages)} stages)" if mesh.feasible else "-",
                     f"{need / MB:.0f} MB" if need else "-"])
        if not mesh.feasible and all(c == "-" for c in cells):
            break
    if not single_max or mesh_max is None:
        raise RuntimeError("no tested size fits a single device or the mesh")
    best_name, (P_single, single_cfg, single_plan) = max(single_max.items(), key=lambda kv: kv[1][0])
    P_mesh, mesh_cfg, mesh_plan = mesh_max
    run_single = _train(single_cfg, single_plan, threads, steps)
    run_mesh = _train(mesh_cfg, mesh_plan, threads, steps)

    def held(run):
        return ", ".join(f"{n}: {h / MB:.0f}/{b / MB:.0f} MB" for n, h, b in run["held"])

    gain = P_mesh / P_single
    penalty = run_single["steps_per_s"] / run_mesh["steps_per_s"]
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
                 [["single device", f"{P_single / 1e6:.1f}M", best_name, f"{run_single['steps_per_s']:.3f}",
                   held(run_single), f"{run_single['loss_first']:.3f} -> {run_single['loss_last']:.3f}"],
                  ["mesh", f"{P_mesh / 1e6:.1f}M", " -> ".join(s.worker_name for s in mesh_plan.stages),
                   f"{run_mesh['steps_per_s']:.3f}", held(run_mesh),
                   f"{run_mesh['loss_first']:.3f} -> {run_mesh['loss_last']:.3f}"]]),
        f"**capacity_gain = {P_mesh / 1e6:.1f}M / {P_single / 1e6:.1f}M = {gain:.2f}x**; throughput penalty "
        f"{penalty:.2f}x (emulated: one core per worker, loopback links - only the capacity ratio is meaningful)."])
    if write_doc:
        update_section("capacity-emulated", md)
    return md


def b200_capacity(write_doc: bool = True) -> str:
    """Largest Llama-family model (d=4096 blocks, seq 4096) per number of B200s, planner-only."""
    from meshtrain_b200.api import plan_device_pipeline

    rows = []
    for gpus in (1, 2, 4, 8):
        for offload in (False, True):
            best = None
            for blocks in range(4, 161, 4):
                cfg = {"type": "llama", "layers": blocks, "hidden_size": 4096, "heads": 32, "n_kv_heads": 8,
                       "ffn_hidden": 14336, "vocab_size": 128256, "seq_len": 4096, "dtype": "bfloat16"}
                spec = build_model_spec(cfg)
                if gpus > spec.num_layers:
                    continue
                try:
                    plan_device_pipeline(spec, gpus, 32, 1, "1f1b", "adam", offload=offload, memory_gb=180.0)
                except RuntimeError:
                    break
                best = (blocks, spec.parameter_count())
            rows.append([gpus, "host" if offload else "device", f"{best[0]} blocks" if best else "-",
                         f"{best[1] / 1e9:.1f} B" if best else "-"])
    md = "\n\n".join([environment_line(), "Planner-only: largest Llama-style model (d 4096, GQA 32/8, SwiGLU 14336, "
                      "seq 4096, 32 microbatches of 1, Adam, bf16 compute + fp32 master) that fits N B200s "
                      "(180 GB each) with fp32 master weights + Adam moments on the device or offloaded to host DRAM.",
                      md_table(["B200s", "optimizer state", "largest model", "parameters"], rows)])
    if write_doc:
        update_section("capacity-b200", md)
    return md


def run_hardware(client, sizes=SIZES, steps: int = 5, write_doc: bool = True, poll_s: float = 1.0) -> str:
    workers = [w for w in client.status()["workers"] if w["status"] == "ONLINE"]
    if len(workers) < 2:
        raise ValueError("the hardware capacity comparison needs at least two online workers")

    def submit(cfg_model, *, alone: str | None = None):
        cfg = {"job": {"name": "capacity"}, "model": cfg_model,
               "training": {"batch_size": BATCH, "microbatch_size": MICRO, "learning_rate": 3e-4,
                            "optimizer": "adamw", "steps": steps, "log_every": 1},
               "placement": {"strategy": "auto", "num_stages": len(workers), "enforce_memory_check": True},
               "network": {"timeout_s": 300}}
        if alone:
            n = build_model_spec(cfg_model).num_layers
            cfg["placement"] = {"strategy": "manual", "enforce_memory_check": False,
                                "stages": [{"worker": alone, "layers": [0, n]}]}
        try:
            job = client.start_job(cfg)
        except Exception as exc:  # noqa: BLE001 - a refused plan is a failed size
            return {"ok": False, "error": str(exc)[:200]}
        while (j := client.job(job["job_id"]))["status"] == "RUNNING":
            time.sleep(poll_s)
        ok = j["status"] == "COMPLETED"
        s = j.get("summary") or {}
        return {"ok": ok, "error": j.get("error"), "stages": len(j["stage_workers"]),
                "steps_per_s": 1 / s["mean_step_s"] if ok and s.get("mean_step_s") else None}

    single = {w["worker_id"]: {} for w in workers}
    mesh: dict = {}
    for blocks, hidden in sizes:
        cfg = model_cfg(blocks, hidden)
        P = build_model_spec(cfg).parameter_count()
        for wid, rec in single.items():
            if rec.get("failed"):
                continue
            r = submit(cfg, alone=wid)
            rec.update({"max_P": P, "steps_per_s": r["steps_per_s"]} if r["ok"] else {"failed": r["error"]})
        if not mesh.get("failed"):
            r = submit(cfg)
            mesh.update({"max_P": P, "steps_per_s": r["steps_per_s"], "stages": r["stages"]} if r["ok"]
                        else {"failed": r["error"]})
        if mesh.get("failed") and all(v.get("failed") for v in single.values()):
            break

    def clean(err):
        return (err or "").replace("\n", " ").replace("|", "/")[:120]

    rows = [[wid, f"{v.get('max_P', 0) / 1e6:.1f}M", f"{v.get('steps_per_s') or 0:.3f}",
             1 if "max_P" in v else "-", clean(v.get("failed"))] for wid, v in single.items()]
    rows.append(["mesh", f"{mesh.get('max_P', 0) / 1e6:.1f}M", f"{mesh.get('steps_per_s') or 0:.3f}",
                 mesh.get("stages", "-"), clean(mesh.get("failed"))])
    best = max((v for v in single.values() if "max_P" in v), key=lambda v: v["max_P"], default=None)
    parts = [environment_line(), f"**Mode: hardware** (real devices through the coordinator); mesh trials use all "
             f"{len(workers)} online workers. P_max is the largest size that trained.",
             md_table(["device", "P_max", "steps/s at P_max", "stages", "first failure"], rows)]
    if best and mesh.get("max_P"):
        parts.append(f"capacity_gain = {mesh['max_P'] / best['max_P']:.2f}x, throughput penalty = "
                     f"{(best['steps_per_s'] or 0) / (mesh['steps_per_s'] or 1):.2f}x")
    md = "\n\n".join(parts)
    if write_doc:
        update_section("capacity-hardware", md)
    return md


def run_experiment5(mode: str = "emulated", cluster_file: str | None = None, steps: int = 5, *, client=None) -> str:
    if mode == "emulated":
        return run_emulated(steps=steps)
    if mode == "b200":
        return b200_capacity()
    if client is None:
        from meshtrain_b200.cli import client_from

        client = client_from()
    try:
        return run_hardware(client, steps=steps)
    finally:
        client.close()

"""Placement strategies compared: equal vs compute-aware vs memory+compute+network-aware.

Three sources of a cluster (reference experiments/placement.py:1-105):

* ``cluster_file`` - JSON written by ``meshtrain cluster benchmark --output``:
  plans for that measured cluster (predictions only);
* ``b200`` - one 8 x B200 box (NVLink links, 180 GB each) for the GPT and
  Llama configurations (predictions only);
* default - emulated CPU workers on this host; every plan is also trained and
  its measured step time and held memory are reported.
"""

from __future__ import annotations

import json
import statistics

from meshtrain_b200.experiments.emulation import MB, EmulatedWorker, profile_emulated
from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.planner.cost import NetworkModel
from meshtrain_b200.planner.graph import analytic_profile, profile_model
from meshtrain_b200.planner.partition import PlannerOptions, WorkerProfile, b200_box, make_plan

MODEL = {"type": "tiny_transformer", "layers": 10, "hidden_size": 256, "heads": 4, "vocab_size": 512, "seq_len": 64}
BATCH, MICRO = 16, 4
WORKERS = [EmulatedWorker("fast-small", threads=2, memory_budget_bytes=90 * MB, label="2 threads, 90 MB"),
           EmulatedWorker("slow-large", threads=1, memory_budget_bytes=260 * MB, label="1 thread, 260 MB"),
           EmulatedWorker("slow-mid", threads=1, memory_budget_bytes=150 * MB, label="1 thread, 150 MB")]
STRATEGIES = ("equal", "compute", "topology_aware")


def _opts(n_mb: int, num_stages: int | None = None) -> PlannerOptions:
    return PlannerOptions(optimizer="adamw", num_microbatches=n_mb, headroom_fraction=0.1, headroom_min_bytes=4 * MB,
                          num_stages=num_stages)


def _placement(plan) -> str:
    return " / ".join(f"{s.worker_name}:{s.start}-{s.end - 1}" for s in plan.stages)


def _measure(plan, by_name: dict[str, EmulatedWorker], steps: int) -> dict:
    stages = [LocalStage((s.start, s.end), "cpu", threads=by_name[s.worker_id].threads) for s in plan.stages]
    settings = PipelineSettings("placement", steps=steps, batch_size=BATCH, num_microbatches=BATCH // MICRO,
                                log_every=1000)
    res = run_local_pipeline(MODEL, stages, settings, optimizer="adamw", lr=3e-4)
    step_s = statistics.median(m["step_s"] for m in res[0].step_metrics[2:] or res[0].step_metrics)
    held = {}
    for r in res:
        m = r.step_metrics[-1]["memory"]
        held[r.stage_index] = m["parameters"] + m["gradients"] + m["optimizer_state"] + m["saved_activations_peak"]
    return {"step_s": step_s, "held": held, "loss_first": res[0].losses[0], "loss_last": res[0].losses[-1]}


def b200_plans() -> str:
    """Planner predictions for the GPT / Llama configurations on one 8 x B200 box."""
    from meshtrain_b200.api import plan_device_pipeline

    cases = [("gpt-0.48b", {"type": "gpt", "layers": 24, "hidden_size": 1280, "heads": 20, "vocab_size": 50257,
                            "seq_len": 2048, "dtype": "bfloat16"}, 32, 4, [1, 2, 4, 8], False),
             ("llama-8b", {"type": "llama", "layers": 32, "hidden_size": 4096, "heads": 32, "n_kv_heads": 8,
                           "ffn_hidden": 14336, "vocab_size": 128256, "seq_len": 4096, "dtype": "bfloat16"},
              64, 1, [4, 8], False),
             ("llama-8b + offload", {"type": "llama", "layers": 32, "hidden_size": 4096, "heads": 32,
                                     "n_kv_heads": 8, "ffn_hidden": 14336, "vocab_size": 128256, "seq_len": 4096,
                                     "dtype": "bfloat16"}, 32, 1, [4], True)]
    rows = []
    for name, cfg, M, mbs, ns, off in cases:
        spec = build_model_spec(cfg)
        for n in ns:
            try:
                p = plan_device_pipeline(spec, n, M, mbs, "1f1b", "adam", offload=off, memory_gb=180.0)
                rows.append([name, n, " / ".join(f"{a}-{b - 1}" for a, b in p.ranges()),
                             f"{max(s.memory.required for s in p.stages) / 1024 ** 3:.0f} GB",
                             f"{p.predicted_step_s * 1e3:.0f}"])
            except RuntimeError:
                rows.append([name, n, "does not fit", "-", "-"])
    return md_table(["model", "GPUs", "stage layers", "max stage memory", "predicted ms/step"], rows)


def run_experiment4(cluster_file: str | None = None, steps: int = 12, write_doc: bool = True,
                    b200: bool = False) -> str:
    spec = build_model_spec(MODEL)
    layers = profile_model(spec, MICRO)
    n_mb = BATCH // MICRO
    sections = [environment_line()]
    if b200:
        sections += ["One 8 x B200 box, NVLink links between every pair, device-engine memory accounting "
                     "(predictions only).", b200_plans()]
        tag = "b200"
    elif cluster_file:
        with open(cluster_file) as f:
            bench = json.load(f)
        profiles = [WorkerProfile(w, w, r["backend"], int(r.get("memory_total", 8 * 1024 ** 3)), r["measured_flops"])
                    for w, r in bench["workers"].items()]
        network = NetworkModel.from_measurements(bench.get("links", {}))
        rows = []
        for strat in STRATEGIES:
            p = make_plan(strat, layers, profiles, network, _opts(n_mb))
            rows.append([strat, _placement(p), "yes" if p.feasible else "NO", f"{p.predicted_step_s * 1e3:.1f}",
                         f"{p.communication_bytes_per_step / 1e6:.2f}"])
        sections += [f"Cluster from `{cluster_file}` (predictions only).",
                     md_table(["strategy", "placement", "feasible", "predicted ms/step", "MB/step"], rows)]
        tag = "cluster"
    else:
        profiles = profile_emulated(WORKERS)
        by_name = {w.name: w for w in WORKERS}
        sections.append(f"Emulated CPU workers on one host (compute differences measured, memory budgets declared). "
                        f"Model: tiny transformer ({spec.parameter_count() / 1e6:.2f}M params, {spec.num_layers} "
                        f"layers), AdamW, batch {BATCH}, {n_mb} microbatches, {steps} steps per plan.")
        sections.append(md_table(["worker", "emulated as", "measured GFLOP/s", "compute score"],
                                 [[p.name, by_name[p.name].label, f"{p.measured_flops / 1e9:.1f}",
                                   f"{p.compute_score:.2f}"] for p in profiles]))
        rows = []
        for strat in STRATEGIES:
            p = make_plan(strat, layers, profiles, NetworkModel(),
                          _opts(n_mb, num_stages=3 if strat != "topology_aware" else None))
            m = _measure(p, by_name, steps)
            within = all(m["held"][s.stage_index] <= s.memory.budget for s in p.stages)
            rows.append([strat, _placement(p), "yes" if p.feasible else "NO: " + "; ".join(p.violations),
                         f"{p.predicted_step_s * 1e3:.1f}", f"{m['step_s'] * 1e3:.1f}",
                         " / ".join(f"{m['held'][s.stage_index] / MB:.1f}/{s.memory.budget / MB:.0f}"
                                    for s in p.stages) + (" ok" if within else " EXCEEDED"),
                         f"{m['loss_first']:.3f} -> {m['loss_last']:.3f}"])
        sections.append(md_table(["strategy", "placement (worker:layers)", "memory-feasible", "predicted ms/step",
                                  "measured ms/step", "MB held/budget per stage", "loss"], rows))
        tag = "emulated"
    md = "\n\n".join(sections)
    if write_doc:
        update_section(f"experiment4-{tag}", md)
    return md

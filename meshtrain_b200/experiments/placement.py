"""Placement strategies compared: equal vs compute-aware vs memory+compute+network-aware.

The reference's experiment 4 (experiments/placement.py:1-105) on three kinds of cluster:

* ``cluster_file`` - JSON written by ``meshtrain cluster benchmark --output``:
  plans for that measured cluster (predictions only);
* ``b200`` - one 8 x B200 box (NVLink links, 180 GB each) for the GPT and
  Llama configurations (predictions only);
* default - emulated CPU workers on this host; every plan is also trained and
  its measured step time and held memory are reported.

Every kind goes through ``compare``: plan the model with each strategy for one set of
worker profiles and links, then (emulated workers only) train each plan and put the
measurement beside the prediction.
"""

from __future__ import annotations

import json
import statistics
from dataclasses import dataclass

from meshtrain_b200.experiments.emulation import MB, EmulatedWorker, profile_emulated
from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.planner.cost import NetworkModel
from meshtrain_b200.planner.graph import profile_model
from meshtrain_b200.planner.partition import PlannerOptions, WorkerProfile, make_plan

MODEL = {"type": "tiny_transformer", "layers": 10, "hidden_size": 256, "heads": 4, "vocab_size": 512, "seq_len": 64}
BATCH, MICRO = 16, 4
STRATEGIES = ("equal", "compute", "topology_aware")
# (name, torch threads, memory budget in MB): a fast worker with little memory and two slower,
# larger ones, so the three strategies disagree
_EMULATED = (("fast-small", 2, 90), ("slow-large", 1, 260), ("slow-mid", 1, 150))
WORKERS = [EmulatedWorker(name, threads=t, memory_budget_bytes=mb * MB, label=f"{t} thread{'s' * (t > 1)}, {mb} MB")
           for name, t, mb in _EMULATED]


@dataclass
class Trial:
    strategy: str
    plan: object
    measured: dict | None = None

    @property
    def placement(self) -> str:
        return " / ".join(f"{st.worker_name}:{st.start}-{st.end - 1}" for st in self.plan.stages)

    def within_budgets(self) -> bool:
        held = self.measured["held"]
        return all(held[st.stage_index] <= st.memory.budget for st in self.plan.stages)


def _options(microbatches: int, stages: int | None = None) -> PlannerOptions:
    return PlannerOptions(optimizer="adamw", num_microbatches=microbatches, headroom_fraction=0.1,
                          headroom_min_bytes=4 * MB, num_stages=stages)


def _train(plan, threads_of: dict[str, int], steps: int) -> dict:
    """Runs a plan as CPU processes: median step time (first two steps left out), bytes held, losses."""
    stages = [LocalStage((st.start, st.end), "cpu", threads=threads_of[st.worker_id]) for st in plan.stages]
    settings = PipelineSettings("placement", steps=steps, batch_size=BATCH, num_microbatches=BATCH // MICRO,
                                log_every=1000)
    results = run_local_pipeline(MODEL, stages, settings, optimizer="adamw", lr=3e-4)
    steady = results[0].step_metrics[2:] or results[0].step_metrics
    held = {}
    for res in results:
        mem = res.step_metrics[-1]["memory"]
        held[res.stage_index] = sum(mem[k] for k in ("parameters", "gradients", "optimizer_state",
                                                     "saved_activations_peak"))
    return {"step_s": statistics.median(rec["step_s"] for rec in steady), "held": held,
            "losses": (results[0].losses[0], results[0].losses[-1])}


def compare(layers, profiles, network, microbatches: int, *, stages_for=lambda strategy: None,
            measure=None) -> list[Trial]:
    """One plan per strategy; ``measure(plan)`` (if given) trains it and returns its figures."""
    trials = [Trial(s, make_plan(s, layers, profiles, network, _options(microbatches, stages_for(s))))
              for s in STRATEGIES]
    if measure is not None:
        for trial in trials:
            trial.measured = measure(trial.plan)
    return trials


def b200_plans() -> str:
    """Planner predictions for the GPT / Llama configurations on one 8 x B200 box."""
    from meshtrain_b200.api import plan_device_pipeline

    llama = {"type": "llama", "layers": 32, "hidden_size": 4096, "heads": 32, "n_kv_heads": 8, "ffn_hidden": 14336,
             "vocab_size": 128256, "seq_len": 4096, "dtype": "bfloat16"}
    gpt = {"type": "gpt", "layers": 24, "hidden_size": 1280, "heads": 20, "vocab_size": 50257, "seq_len": 2048,
           "dtype": "bfloat16"}
    # (label, model, microbatches, microbatch size, GPU counts, offload)
    cases = (("gpt-0.48b", gpt, 32, 4, (1, 2, 4, 8), False), ("llama-8b", llama, 64, 1, (4, 8), False),
             ("llama-8b + offload", llama, 32, 1, (4,), True))
    rows = []
    for label, cfg, microbatches, mbs, gpu_counts, offload in cases:
        spec = build_model_spec(cfg)
        for gpus in gpu_counts:
            try:
                plan = plan_device_pipeline(spec, gpus, microbatches, mbs, "1f1b", "adam", offload=offload,
                                            memory_gb=180.0)
            except RuntimeError:
                rows.append([label, gpus, "does not fit", "-", "-"])
                continue
            worst = max(st.memory.required for st in plan.stages)
            rows.append([label, gpus, " / ".join(f"{a}-{b - 1}" for a, b in plan.ranges()),
                         f"{worst / 1024 ** 3:.0f} GB", f"{plan.predicted_step_s * 1e3:.0f}"])
    return md_table(["model", "GPUs", "stage layers", "max stage memory", "predicted ms/step"], rows)


def _profiles_from_file(path: str) -> tuple[list[WorkerProfile], NetworkModel]:
    with open(path) as f:
        bench = json.load(f)
    profiles = [WorkerProfile(wid, wid, rec["backend"], int(rec.get("memory_total", 8 * 1024 ** 3)),
                              rec["measured_flops"]) for wid, rec in bench["workers"].items()]
    return profiles, NetworkModel.from_measurements(bench.get("links", {}))


def run_experiment4(cluster_file: str | None = None, steps: int = 12, write_doc: bool = True,
                    b200: bool = False) -> str:
    spec = build_model_spec(MODEL)
    layers = profile_model(spec, MICRO)
    microbatches = BATCH // MICRO
    sections = [environment_line()]
    if b200:
        tag = "b200"
        sections += ["One 8 x B200 box, NVLink links between every pair, device-engine memory accounting "
                     "(predictions only).", b200_plans()]
    elif cluster_file:
        tag = "cluster"
        profiles, network = _profiles_from_file(cluster_file)
        trials = compare(layers, profiles, network, microbatches)
        sections += [f"Cluster from `{cluster_file}` (predictions only).",
                     md_table(["strategy", "placement", "feasible", "predicted ms/step", "MB/step"],
                              [[t.strategy, t.placement, "yes" if t.plan.feasible else "NO",
                                f"{t.plan.predicted_step_s * 1e3:.1f}",
                                f"{t.plan.communication_bytes_per_step / 1e6:.2f}"] for t in trials])]
    else:
        tag = "emulated"
        profiles = profile_emulated(WORKERS)
        label_of = {w.name: w.label for w in WORKERS}
        threads_of = {w.name: w.threads for w in WORKERS}
        # equal and compute-aware split over all three workers; the topology-aware planner chooses its stage count
        trials = compare(layers, profiles, NetworkModel(), microbatches,
                         stages_for=lambda s: None if s == "topology_aware" else 3,
                         measure=lambda plan: _train(plan, threads_of, steps))
        sections += [
            f"Emulated CPU workers on one host (compute differences measured, memory budgets declared). Model: tiny "
            f"transformer ({spec.parameter_count() / 1e6:.2f}M params, {spec.num_layers} layers), AdamW, batch "
            f"{BATCH}, {microbatches} microbatches, {steps} steps per plan.",
            md_table(["worker", "emulated as", "measured GFLOP/s", "compute score"],
                     [[p.name, label_of[p.name], f"{p.measured_flops / 1e9:.1f}", f"{p.compute_score:.2f}"]
                      for p in profiles])]
        rows = []
        for t in trials:
            m = t.measured
            budgets = " / ".join(f"{m['held'][st.stage_index] / MB:.1f}/{st.memory.budget / MB:.0f}"
                                 for st in t.plan.stages)
            rows.append([t.strategy, t.placement,
                         "yes" if t.plan.feasible else "NO: " + "; ".join(t.plan.violations),
                         f"{t.plan.predicted_step_s * 1e3:.1f}", f"{m['step_s'] * 1e3:.1f}",
                         budgets + (" ok" if t.within_budgets() else " EXCEEDED"),
                         f"{m['losses'][0]:.3f} -> {m['losses'][1]:.3f}"])
        sections.append(md_table(["strategy", "placement (worker:layers)", "memory-feasible", "predicted ms/step",
                                  "measured ms/step", "MB held/budget per stage", "loss"], rows))
    md = "\n\n".join(sections)
    if write_doc:
        update_section(f"experiment4-{tag}", md)
    return md

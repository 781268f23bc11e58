"""Tiny transformer, 3 stages over loopback TCP, microbatched (reference experiments/transformer.py:1-55).

One-step gradient equivalence, then training compared step by step with the
single-process loss trajectory on the same data.
"""

from __future__ import annotations

from meshtrain_b200.experiments.correctness import run_gradient_equivalence
from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, reference_step, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.summary import summarize

MODEL = {"type": "tiny_transformer", "layers": 6, "hidden_size": 128, "heads": 4, "vocab_size": 128, "seq_len": 32}
STAGES = [LocalStage((0, 3)), LocalStage((3, 5)), LocalStage((5, 8))]


def run_experiment_transformer(steps: int = 150, write_doc: bool = True) -> str:
    spec = build_model_spec(MODEL)
    rows, _ = run_gradient_equivalence(MODEL, STAGES, batch_size=16, num_microbatches=4, transport="tcp")
    worst = max(rows, key=lambda r: r.relative)
    settings = PipelineSettings("transformer", steps=steps, batch_size=16, num_microbatches=4, log_every=10 ** 6)
    res = run_local_pipeline(MODEL, STAGES, settings, optimizer="adamw", lr=1e-3, transport="tcp", capture_params=True)
    ref, _, _ = reference_step(MODEL, settings, optimizer="adamw", lr=1e-3, steps=steps)
    losses = res[0].losses
    dev = max(abs(a - b) / max(abs(b), 1e-8) for a, b in zip(losses, ref))
    s = summarize([m for r in res for m in r.step_metrics])
    changed = all(all(not (r.initial_params[k] == r.final_params[k]).all() for k in r.initial_params) for r in res)
    curve = [[i, f"{losses[i]:.4f}", f"{ref[i]:.4f}"] for i in sorted({0, 25, 50, 100, steps - 1}) if i < steps]
    md = "\n\n".join([
        environment_line(),
        f"CPU, 3 stage processes over loopback TCP. Model {spec.parameter_count() / 1e6:.2f}M params "
        f"({spec.num_layers} layers), stages {[s.layers for s in STAGES]}, batch 16 = 4 microbatches, AdamW lr 1e-3.",
        f"- one-step gradient equivalence: max relative error {worst.relative:.2e} ({worst.name})",
        f"- training: loss {losses[0]:.4f} -> {losses[-1]:.4f} over {steps} steps; every stage updated: {changed}; "
        f"max relative deviation from the single-process curve: {dev:.2e}",
        f"- throughput: {s['mean_step_s'] * 1e3:.1f} ms/step, {s['bytes_per_step'] / 1e6:.3f} MB sent per step",
        md_table(["step", "pipeline loss", "single-process loss"], curve)])
    if write_doc:
        update_section("transformer-3-stages", md)
    return md

"""The tiny-Transformer milestone and correctness gate: 3 CPU stage processes over TCP.

Shape (``configs/c1_tiny_transformer_cpu.yaml``): decoder-only Transformer,
vocab 1024, d_model 128, 4 blocks of 4 heads, MLP 512, GELU, pre-LayerNorm,
learned positions, sequences of 64 tokens drawn i.i.d. uniform from seed 0
with next-token targets; batch 8 as 4 microbatches; Adam, lr 1e-3; fp32.

``run_c1_gate`` runs the model as three stage processes on loopback TCP under
GPipe and under 1F1B and compares every step's loss with the single-process
oracle on the same data (``reference_step``).  The gate is a relative loss
deviation of at most ``C1_TOLERANCE`` (2e-7).  Every process, the oracle
included, uses one torch thread, so the CPU kernels sum in the same order.
``run_experiment_transformer`` writes the result as a results section, followed by
the reference's own milestone on its own shape (``run_milestone``: the 1.23M-parameter
model on arithmetic sequences, 3 TCP stages, batch 16 as 4 microbatches, AdamW): a
one-step gradient comparison, then the loss curve against one process and the
throughput (reference experiments/transformer.py:16-55; its docs/v1-results.md:253-259
report 61.2 ms/step and 2.35e-7 loss deviation over 150 steps).
"""

from __future__ import annotations

import torch

from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, reference_step, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.summary import summarize

C1_MODEL = {"type": "tiny_transformer", "layers": 4, "hidden_size": 128, "heads": 4, "vocab_size": 1024,
            "seq_len": 64, "dtype": "float32", "data": "uniform"}
C1_TOLERANCE = 2e-7
BATCH, MICROBATCHES, LR = 8, 4, 1e-3


def c1_stages() -> list[LocalStage]:
    """Three contiguous stages over the model's layers (embedding, 4 blocks, head)."""
    n = build_model_spec(C1_MODEL).num_layers
    return [LocalStage((n * i // 3, n * (i + 1) // 3)) for i in range(3)]


def run_c1_gate(schedule: str, steps: int = 10) -> dict:
    """Loss curve of the 3-stage TCP pipeline vs. one process, for one schedule."""
    settings = PipelineSettings(f"c1-{schedule}", steps=steps, batch_size=BATCH, num_microbatches=MICROBATCHES,
                                schedule=schedule, async_transport=True, log_every=10 ** 6)
    stages = c1_stages()
    results = run_local_pipeline(C1_MODEL, stages, settings, optimizer="adam", lr=LR, transport="tcp",
                                 torch_threads=1)
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        oracle, _, _ = reference_step(C1_MODEL, settings, optimizer="adam", lr=LR, steps=steps)
    finally:
        torch.set_num_threads(threads)
    losses = results[0].losses
    deviation = max(abs(a - b) / abs(b) for a, b in zip(losses, oracle))
    return {"schedule": schedule, "steps": steps, "losses": losses, "oracle": oracle, "max_rel_deviation": deviation,
            "passed": len(losses) == steps and deviation <= C1_TOLERANCE,
            "summary": summarize([m for r in results for m in r.step_metrics]),
            "stages": [s.layers for s in stages]}


MILESTONE_MODEL = {"type": "tiny_transformer", "layers": 6, "hidden_size": 128, "heads": 4, "vocab_size": 128,
                   "seq_len": 32}
MILESTONE_SPLIT = [(0, 3), (3, 5), (5, 8)]


def run_milestone(steps: int = 150) -> dict:
    """The reference's milestone-8 run: gradients of one step, then ``steps`` steps against one process."""
    from meshtrain_b200.experiments.correctness import run_gradient_equivalence

    stages = [LocalStage(r) for r in MILESTONE_SPLIT]
    grad_rows, _ = run_gradient_equivalence(MILESTONE_MODEL, stages, batch_size=16, num_microbatches=4,
                                            transport="tcp")
    settings = PipelineSettings("milestone", steps=steps, batch_size=16, num_microbatches=4, log_every=10 ** 6)
    results = run_local_pipeline(MILESTONE_MODEL, stages, settings, optimizer="adamw", lr=1e-3, transport="tcp")
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        oracle, _, _ = reference_step(MILESTONE_MODEL, settings, optimizer="adamw", lr=1e-3, steps=steps)
    finally:
        torch.set_num_threads(threads)
    losses = results[0].losses
    return {"worst_gradient": max(grad_rows, key=lambda r: r.relative), "gradients": len(grad_rows),
            "losses": losses, "oracle": oracle,
            "max_rel_deviation": max(abs(a - b) / max(abs(b), 1e-8) for a, b in zip(losses, oracle)),
            "summary": summarize([m for r in results for m in r.step_metrics])}


def _milestone_section(m: dict, steps: int) -> str:
    spec = build_model_spec(MILESTONE_MODEL)
    worst, s = m["worst_gradient"], m["summary"]
    marks = sorted(i for i in {0, 25, 50, 100, steps - 1} if i < steps)
    return "\n\n".join([
        f"Milestone on the reference's own shape: {spec.parameter_count() / 1e6:.2f}M params ({spec.num_layers} "
        f"layers), stages {MILESTONE_SPLIT}, batch 16 = 4 microbatches, AdamW 1e-3, arithmetic sequences, TCP.",
        f"- One-step gradients: worst relative error {worst.relative:.2e} ({worst.name}) over {m['gradients']} tensors\n"
        f"- {steps} steps: loss {m['losses'][0]:.4f} -> {m['losses'][-1]:.4f}; max relative deviation from one "
        f"process {m['max_rel_deviation']:.2e}\n"
        f"- Throughput: {s['mean_step_s'] * 1e3:.1f} ms/step, {16 / s['mean_step_s']:.1f} samples/s, "
        f"{s['bytes_per_step'] / 1e6:.3f} MB sent per step",
        md_table(["step", "pipeline loss", "single-process loss"],
                 [[i, f"{m['losses'][i]:.4f}", f"{m['oracle'][i]:.4f}"] for i in marks])])


def run_experiment_transformer(steps: int = 150, write_doc: bool = True) -> str:
    runs = [run_c1_gate(schedule, steps) for schedule in ("gpipe", "1f1b")]
    spec = build_model_spec(C1_MODEL)
    rows = [[r["schedule"], f"{r['losses'][0]:.5f} -> {r['losses'][-1]:.5f}", f"{r['max_rel_deviation']:.2e}",
             "pass" if r["passed"] else "FAIL", f"{r['summary']['mean_step_s'] * 1e3:.1f}",
             f"{r['summary']['bytes_per_step'] / 1e6:.3f}"] for r in runs]
    md = "\n\n".join([
        environment_line(),
        f"CPU, 3 stage processes over loopback TCP, one torch thread each. Model {spec.parameter_count() / 1e6:.2f}M "
        f"params ({spec.num_layers} layers), stages {runs[0]['stages']}, batch {BATCH} = {MICROBATCHES} microbatches, "
        f"uniform tokens, Adam lr {LR:g}, {steps} steps; gate: loss within {C1_TOLERANCE:g} (relative) of one process.",
        md_table(["schedule", "loss first -> last", "max rel. deviation", "gate", "ms/step", "MB/step"], rows),
        _milestone_section(run_milestone(steps), steps)])
    if write_doc:
        update_section("transformer-3-stages", md)
    return md

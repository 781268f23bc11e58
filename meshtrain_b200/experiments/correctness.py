"""Gradient equivalence: pipelined stages vs. the whole model in one process.

One training step runs twice on the same seeds and batches: once through
``run_local_pipeline`` (one OS process per stage, tensors crossing process
boundaries as framed packets) and once through ``reference_step``.  Each
parameter's gradient is compared by max/mean absolute error and by relative
L2 error (reference experiments/correctness.py:1-104).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from meshtrain_b200.parallel.local import LocalStage, global_param_names, reference_step, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings


@dataclass
class GradientError:
    name: str
    stage: int
    max_abs: float
    mean_abs: float
    relative: float  # ||g_pipe - g_ref||_2 / ||g_ref||_2 (max_abs when g_ref == 0)


def compare_gradients(reference: dict[str, torch.Tensor], distributed: dict[str, torch.Tensor],
                      stage_of: dict[str, int] | None = None) -> list[GradientError]:
    diff_names = set(reference) ^ set(distributed)
    if diff_names:
        raise AssertionError(f"gradient sets differ: {sorted(diff_names)}")
    out = []
    for name, ref in reference.items():
        r = ref.detach().to(torch.float64).cpu()
        d = distributed[name].detach().to(torch.float64).cpu()
        err = d - r
        norm = float(r.norm())
        max_abs = float(err.abs().max()) if err.numel() else 0.0
        out.append(GradientError(name, (stage_of or {}).get(name, -1), max_abs,
                                 float(err.abs().mean()) if err.numel() else 0.0,
                                 float(err.norm()) / norm if norm > 0 else max_abs))
    return out


def format_gradient_report(rows: list[GradientError]) -> str:
    head = f"{'parameter':<30}{'stage':>6}{'max_abs':>12}{'mean_abs':>12}{'relative':>12}"
    body = [f"{r.name:<30}{r.stage:>6}{r.max_abs:>12.2e}{r.mean_abs:>12.2e}{r.relative:>12.2e}" for r in rows]
    return "\n".join([head, "-" * len(head), *body])


def run_gradient_equivalence(model_cfg: dict, stages: list[LocalStage], *, batch_size: int = 32,
                             num_microbatches: int = 1, seed: int = 0, transport: str = "pipe",
                             schedule: str = "gpipe", reference_device: str = "cpu"
                             ) -> tuple[list[GradientError], dict]:
    settings = PipelineSettings(job_id="grad-equivalence", steps=1, batch_size=batch_size,
                                num_microbatches=num_microbatches, capture_gradients_at_step=0, log_every=1,
                                schedule=schedule)
    ref_losses, ref_grads, _ = reference_step(model_cfg, settings, seed=seed, device=reference_device)
    results = run_local_pipeline(model_cfg, stages, settings, seed=seed, transport=transport)
    grads: dict[str, torch.Tensor] = {}
    stage_of: dict[str, int] = {}
    for res in results:
        g = global_param_names(stages, res.gradients, res.stage_index)
        grads.update(g)
        stage_of.update(dict.fromkeys(g, res.stage_index))
    rows = compare_gradients(ref_grads, grads, stage_of)
    info = {"reference_loss": ref_losses[0], "distributed_loss": results[0].losses[0],
            "stages": [list(s.layers) for s in stages], "devices": [s.device for s in stages],
            "transport": transport, "microbatches": num_microbatches, "schedule": schedule}
    return rows, info


_CASES = [
    ("MLP, 2 stages", {"type": "mlp"}, [(0, 3), (3, 7)], 32, 1),
    ("MLP, 3 stages", {"type": "mlp"}, [(0, 2), (2, 5), (5, 7)], 32, 1),
    ("MLP, 2 stages, 4 microbatches", {"type": "mlp"}, [(0, 3), (3, 7)], 32, 4),
    ("tiny transformer (4 blocks, d=64), 3 stages, 2 microbatches",
     {"type": "tiny_transformer", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 64, "seq_len": 16},
     [(0, 2), (2, 4), (4, 6)], 8, 2),
]


def run_experiment1(transport: str = "pipe", write_doc: bool = True, tolerance: float = 1e-4) -> str:
    """CPU stages in separate processes vs. one process; returns the markdown table."""
    from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section

    table, notes = [], []
    for title, cfg, ranges, bs, mbs in _CASES:
        stages = [LocalStage(r) for r in ranges]
        rows, info = run_gradient_equivalence(cfg, stages, batch_size=bs, num_microbatches=mbs, transport=transport)
        worst = max(rows, key=lambda r: r.relative)
        table.append([title, transport, len(stages), mbs, len(rows), f"{max(r.max_abs for r in rows):.2e}",
                      f"{worst.relative:.2e}", f"{abs(info['reference_loss'] - info['distributed_loss']):.2e}",
                      "PASS" if worst.relative < tolerance else "FAIL"])
        per_stage: dict[int, float] = {}
        for r in rows:
            per_stage[r.stage] = max(per_stage.get(r.stage, 0.0), r.max_abs)
        notes.append(f"- **{title}**: per-stage max abs error "
                     + ", ".join(f"stage{s} {v:.2e}" for s, v in sorted(per_stage.items())))
    md = "\n\n".join([environment_line(),
                      "CPU only; each stage is its own OS process and tensors cross as framed packets.",
                      md_table(["case", "transport", "stages", "microbatches", "params", "max abs err",
                                "max relative err", "loss abs diff", "result"], table),
                      "\n".join(notes)])
    if write_doc:
        update_section(f"experiment1-{transport}", md)
    return md

"""A pipeline on real devices vs. a CPU single-process reference (reference
experiments/device_correctness.py:1-118).

``devices`` lists one device per stage (``cpu``, ``cuda:0``, ``cuda:1`` ...);
each stage runs in its own process over loopback TCP.  Compared for the same
seeds and data: loss per step, first-step gradients of every parameter,
per-parameter gradient norms per step, first-update parameter deltas, and the
logits of the final weights on a probe batch.  Tolerances are documented, not
bitwise: 1e-5 relative when every stage is on the CPU, 5e-3 with any
accelerator stage (other kernels and reduction orders).
"""

from __future__ import annotations

import torch

from meshtrain_b200.experiments.correctness import compare_gradients
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, global_param_names, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.parallel.stage import build_optimizer

CPU_TOL = 1e-5
ACCEL_TOL = 5e-3
DEFAULT_MODEL = {"type": "tiny_transformer", "layers": 4, "hidden_size": 128, "heads": 4, "vocab_size": 256,
                 "seq_len": 32}


def _rel(a: float, b: float) -> float:
    return abs(a - b) / max(abs(b), 1e-12)


def _reference(model_cfg, settings, optimizer, lr, steps):
    spec = build_model_spec(model_cfg)
    model = spec.build_full()
    opt = build_optimizer(optimizer, model.parameters(), lr)
    M = settings.num_microbatches
    losses, norms, first_grads, deltas = [], [], None, None
    for step in range(steps):
        x, y = spec.make_batch(step, settings.batch_size)
        total = 0.0
        for xm, ym in zip(x.chunk(M), y.chunk(M)):
            loss = spec.loss_fn(model(xm), ym)
            (loss / M).backward()
            total += loss.item()
        losses.append(total / M)
        norms.append({n: float(p.grad.norm()) for n, p in model.named_parameters()})
        if step == 0:
            first_grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
            before = {n: p.detach().clone() for n, p in model.named_parameters()}
        opt.step()
        opt.zero_grad(set_to_none=True)
        if step == 0:
            deltas = {n: float((p.detach() - before[n]).norm()) for n, p in model.named_parameters()}
    return spec, model, losses, norms, first_grads, deltas


def run_device_correctness(devices: list[str], model_cfg: dict | None = None, steps: int = 3, batch_size: int = 8,
                           num_microbatches: int = 4, optimizer: str = "adamw", lr: float = 1e-3,
                           schedule: str = "1f1b") -> dict:
    model_cfg = model_cfg or DEFAULT_MODEL
    n_layers = build_model_spec(model_cfg).num_layers
    k = len(devices)
    stages = [LocalStage((n_layers * i // k, n_layers * (i + 1) // k), d) for i, d in enumerate(devices)]
    settings = PipelineSettings("device-correctness", steps=steps, batch_size=batch_size,
                                num_microbatches=num_microbatches, schedule=schedule, async_transport=True,
                                capture_gradients_at_step=0, correctness_probe_steps=steps)
    res = run_local_pipeline(model_cfg, stages, settings, optimizer=optimizer, lr=lr, transport="tcp",
                             capture_params=True)
    spec, ref_model, ref_losses, ref_norms, ref_grads, ref_deltas = _reference(model_cfg, settings, optimizer, lr,
                                                                               steps)
    grads, final, norms, deltas = {}, {}, [dict() for _ in range(steps)], {}
    for r in res:
        grads.update(global_param_names(stages, r.gradients, r.stage_index))
        final.update(global_param_names(stages, r.final_params, r.stage_index))
        for i, m in enumerate(r.step_metrics[:steps]):
            c = m["correctness"]
            norms[i].update(global_param_names(stages, {n: torch.tensor(v) for n, v in c["grad_norms"].items()},
                                               r.stage_index))
            if "param_delta_norms" in c:
                deltas.update(global_param_names(
                    stages, {n: torch.tensor(v) for n, v in c["param_delta_norms"].items()}, r.stage_index))
    loss_err = max(_rel(a, b) for a, b in zip(res[0].losses, ref_losses))
    grad_err = max(r.relative for r in compare_gradients(ref_grads, grads))
    norm_err = max(_rel(float(norms[i][n]), ref_norms[i][n]) for i in range(steps) for n in ref_norms[i])
    delta_err = max(_rel(float(deltas[n]), ref_deltas[n]) for n in ref_deltas)
    probe_model = spec.build_full()
    probe_model.load_state_dict({n: final[n].to(torch.float32) for n in ref_model.state_dict()})
    x, _ = spec.make_batch(10 ** 6, batch_size)
    with torch.no_grad():
        a, b = probe_model(x), ref_model(x)
    logit_err = float((a - b).abs().max() / b.abs().max().clamp_min(1e-12))
    tol = CPU_TOL if all(d.startswith("cpu") for d in devices) else ACCEL_TOL
    errors = {"loss": loss_err, "gradient": grad_err, "grad_norm": norm_err, "param_delta": delta_err,
              "logits": logit_err}
    return {"devices": devices, "tolerance": tol, "errors": errors, "passed": all(v <= tol for v in errors.values()),
            "losses": res[0].losses, "reference_losses": ref_losses}


def format_device_correctness(r: dict) -> str:
    lines = [f"devices: {' -> '.join(r['devices'])}   tolerance {r['tolerance']:.0e} (relative)"]
    for k, v in r["errors"].items():
        lines.append(f"  {k:<12} {v:.2e}  {'ok' if v <= r['tolerance'] else 'FAIL'}")
    lines.append("PASSED" if r["passed"] else "FAILED")
    return "\n".join(lines)

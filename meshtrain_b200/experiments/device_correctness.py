"""A pipeline whose stages run on real devices, checked against one CPU process.

``devices`` gives one device per stage (``cpu``, ``cuda:0``, ``cuda:1`` ...);
every stage is its own process on loopback TCP.  With the same seeds and data
as the single-process oracle, five quantities are compared: the loss of each
step, every parameter's first-step gradient, every parameter's gradient norm
at each step, the size of the first update of every parameter, and the
logits of the final weights on a fresh probe batch.  Errors are relative;
the tolerance is 2e-7 when every stage is on the CPU (oracle and stages run
single-threaded, so they reduce in the same order) and 5e-3 when any stage is
on an accelerator (other kernels, other summation orders).  This is the
reference's device-correctness check (experiments/device_correctness.py:1-118).
"""

from __future__ import annotations

import torch

from meshtrain_b200.experiments.correctness import compare_gradients
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, global_param_names, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.parallel.stage import build_optimizer

CPU_TOL = 2e-7
ACCEL_TOL = 5e-3
DEFAULT_MODEL = {"type": "tiny_transformer", "layers": 4, "hidden_size": 128, "heads": 4, "vocab_size": 256,
                 "seq_len": 32}


def _rel(a: float, b: float) -> float:
    return abs(a - b) / max(abs(b), 1e-12)


class Oracle:
    """The whole model in one CPU process, recording what the pipeline is compared on."""

    def __init__(self, model_cfg: dict, optimizer: str, lr: float):
        self.spec = build_model_spec(model_cfg)
        self.model = self.spec.build_full()
        self.opt = build_optimizer(optimizer, self.model.parameters(), lr)
        self.losses, self.grad_norms = [], []
        self.first_grads = self.first_deltas = None

    def train(self, steps: int, batch_size: int, microbatches: int) -> "Oracle":
        previous = torch.get_num_threads()
        torch.set_num_threads(1)  # the stage processes run one thread each: same reduction order
        try:
            return self._train(steps, batch_size, microbatches)
        finally:
            torch.set_num_threads(previous)

    def _train(self, steps: int, batch_size: int, microbatches: int) -> "Oracle":
        params = dict(self.model.named_parameters())
        for step in range(steps):
            x, y = self.spec.make_batch(step, batch_size)
            losses = []
            for xm, ym in zip(x.chunk(microbatches), y.chunk(microbatches)):
                loss = self.spec.loss_fn(self.model(xm), ym)
                (loss / microbatches).backward()
                losses.append(loss.item())
            self.losses.append(sum(losses) / microbatches)
            self.grad_norms.append({n: float(p.grad.norm()) for n, p in params.items()})
            before = {n: p.detach().clone() for n, p in params.items()} if step == 0 else None
            if step == 0:
                self.first_grads = {n: p.grad.detach().clone() for n, p in params.items()}
            self.opt.step()
            self.opt.zero_grad(set_to_none=True)
            if before is not None:
                self.first_deltas = {n: float((p.detach() - before[n]).norm()) for n, p in params.items()}
        return self


def _gather(stages, results, steps: int):
    """Model-wide names of the pipeline's captured gradients, final params, grad norms and first deltas."""
    grads, final, deltas = {}, {}, {}
    norms = [dict() for _ in range(steps)]
    for r in results:
        rename = lambda d: global_param_names(stages, d, r.stage_index)  # noqa: E731
        grads.update(rename(r.gradients))
        final.update(rename(r.final_params))
        for i, record in enumerate(r.step_metrics[:steps]):
            probe = record["correctness"]
            norms[i].update(rename({n: torch.tensor(v) for n, v in probe["grad_norms"].items()}))
            if "param_delta_norms" in probe:
                deltas.update(rename({n: torch.tensor(v) for n, v in probe["param_delta_norms"].items()}))
    return grads, final, norms, deltas


def run_device_correctness(devices: list[str], model_cfg: dict | None = None, steps: int = 3, batch_size: int = 8,
                           num_microbatches: int = 4, optimizer: str = "adamw", lr: float = 1e-3,
                           schedule: str = "1f1b") -> dict:
    model_cfg = model_cfg or DEFAULT_MODEL
    n_layers, k = build_model_spec(model_cfg).num_layers, len(devices)
    stages = [LocalStage((n_layers * i // k, n_layers * (i + 1) // k), dev) for i, dev in enumerate(devices)]
    settings = PipelineSettings("device-correctness", steps=steps, batch_size=batch_size,
                                num_microbatches=num_microbatches, schedule=schedule, async_transport=True,
                                capture_gradients_at_step=0, correctness_probe_steps=steps)
    results = run_local_pipeline(model_cfg, stages, settings, optimizer=optimizer, lr=lr, transport="tcp",
                                 capture_params=True)
    oracle = Oracle(model_cfg, optimizer, lr).train(steps, batch_size, num_microbatches)
    grads, final, norms, deltas = _gather(stages, results, steps)
    probe_model = oracle.spec.build_full()
    probe_model.load_state_dict({n: final[n].float() for n in oracle.model.state_dict()})
    x, _ = oracle.spec.make_batch(10 ** 6, batch_size)
    with torch.no_grad():
        mine, theirs = probe_model(x), oracle.model(x)
    errors = {
        "loss": max(_rel(a, b) for a, b in zip(results[0].losses, oracle.losses)),
        "gradient": max(row.relative for row in compare_gradients(oracle.first_grads, grads)),
        "grad_norm": max(_rel(float(norms[i][n]), v) for i in range(steps) for n, v in oracle.grad_norms[i].items()),
        "param_delta": max(_rel(float(deltas[n]), v) for n, v in oracle.first_deltas.items()),
        "logits": float((mine - theirs).abs().max() / theirs.abs().max().clamp_min(1e-12)),
    }
    tol = CPU_TOL if all(d.startswith("cpu") for d in devices) else ACCEL_TOL
    return {"devices": devices, "tolerance": tol, "errors": errors, "passed": max(errors.values()) <= tol,
            "losses": results[0].losses, "reference_losses": oracle.losses}


def format_device_correctness(r: dict) -> str:
    lines = [f"devices: {' -> '.join(r['devices'])}   tolerance {r['tolerance']:.0e} (relative)"]
    lines += [f"  {name:<12} {err:.2e}  {'ok' if err <= r['tolerance'] else 'FAIL'}" for name, err in r["errors"].items()]
    lines.append("PASSED" if r["passed"] else "FAILED")
    return "\n".join(lines)

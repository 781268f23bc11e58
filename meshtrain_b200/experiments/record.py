"""``meshtrain results record RUN_DIR --section NAME``: a finished cluster run as a results section.

The section shows the placement and the hardware of each stage, the run's
loss, step time and traffic, per-stage planned vs. measured memory and time,
and a correctness check: the first ``reference_steps`` steps of the same
config are replayed in one CPU process and the loss curves compared (kernels
on accelerators round differently, so a small deviation is expected).  The
reference's results recorder (experiments/record.py:1-75) has the same role.
"""

from __future__ import annotations

import json
from pathlib import Path

import yaml

from meshtrain_b200.config import parse_config
from meshtrain_b200.experiments.results_doc import md_table, update_section
from meshtrain_b200.parallel.local import reference_step
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.telemetry import read_jsonl


class FinishedRun:
    def __init__(self, run_dir: str):
        self.dir = Path(run_dir)
        self.cfg = parse_config(yaml.safe_load((self.dir / "config.yaml").read_text()))
        self.plan = json.loads((self.dir / "plan.json").read_text())
        self.summary = json.loads((self.dir / "summary.json").read_text())
        with_loss = sorted((r for r in read_jsonl(self.dir / "metrics.jsonl") if "loss" in r), key=lambda r: r["step"])
        self.losses = [r["loss"] for r in with_loss]

    def deviation_from_cpu(self, steps: int) -> tuple[int, float]:
        """(steps compared, max relative loss deviation from a single CPU process)."""
        n = min(steps, len(self.losses))
        t = self.cfg.training
        settings = PipelineSettings("ref", steps=n, batch_size=t.batch_size, num_microbatches=t.num_microbatches)
        cpu, _, _ = reference_step(self.cfg.model_spec_dict(), settings, seed=self.cfg.job.seed,
                                   optimizer=t.optimizer, lr=t.learning_rate, steps=n)
        worst = max((abs(a - b) / max(abs(b), 1e-8) for a, b in zip(self.losses[:n], cpu)), default=float("nan"))
        return n, worst

    def stage_rows(self) -> list[list]:
        rows = []
        for s in self.plan["stages"]:
            measured = self.summary["stages"].get(str(s["stage"]), {})
            rows.append([s["stage"], s["worker"], s["backend"], f"{s['layers'][0]}-{s['layers'][1] - 1}",
                         f"{s['memory']['required'] / 1e9:.2f} / {s['memory']['budget'] / 1e9:.2f}",
                         f"{measured.get('device_peak_bytes', 0) / 1e9:.2f}",
                         *(f"{measured.get(k, 0) * 1e3:.1f}" for k in ("forward_s", "backward_s", "comm_s", "idle_s")),
                         f"{measured.get('bytes_sent', 0) / 1e6:.2f}"])
        return rows


def record_run(run_dir: str, section: str, reference_steps: int = 20, cluster_status: dict | None = None,
               write_doc: bool = True) -> str:
    run = FinishedRun(run_dir)
    compared, deviation = run.deviation_from_cpu(reference_steps)
    spec = run.cfg.build_model_spec()
    devices = {w["worker_id"]: (w.get("device") or {}).get("name", "?") for w in (cluster_status or {}).get("workers", [])}
    hardware = " -> ".join(f"{s['worker']} ({s['backend']}, {devices.get(s['worker_id'], '?')})"
                           for s in run.plan["stages"])
    s, t = run.summary, run.cfg.training
    curve = s.get("loss") or []
    first, last = (curve[0][1], curve[-1][1]) if curve else (float("nan"), float("nan"))
    md = "\n\n".join([
        f"Run `{run.dir.name}` on {hardware}",
        f"Model: {run.cfg.model.type}, {spec.parameter_count() / 1e6:.1f}M params ({spec.num_layers} layers); batch "
        f"{t.batch_size}, {t.num_microbatches} microbatches, {t.optimizer}.",
        md_table(["steps", "loss first -> last", "ms/step", "MB/step",
                  f"max rel. loss deviation vs CPU single process (first {compared} steps)"],
                 [[s["steps"], f"{first:.4f} -> {last:.4f}", f"{(s.get('mean_step_s') or 0) * 1e3:.1f}",
                   f"{s.get('bytes_per_step', 0) / 1e6:.2f}", f"{deviation:.2e}"]]),
        md_table(["stage", "worker", "backend", "layers", "planned GB (need / usable)", "device peak GB", "fwd ms",
                  "bwd ms", "comm ms", "idle ms", "MB sent/step"], run.stage_rows())])
    if write_doc:
        update_section(section, md)
    return md

"""Record a finished cluster run (``runs/<job>``) into the results file (reference experiments/record.py:1-75).

Correctness on real hardware: the first steps of the same config are replayed
in one CPU process and the loss curves compared (accelerator kernels differ
numerically from the CPU, so a small deviation is expected).
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


def record_run(run_dir: str, section: str, reference_steps: int = 20, cluster_status: dict | None = None,
               write_doc: bool = True) -> str:
    run = Path(run_dir)
    cfg = parse_config(yaml.safe_load((run / "config.yaml").read_text()))
    plan = json.loads((run / "plan.json").read_text())
    summary = json.loads((run / "summary.json").read_text())
    recs = [r for r in read_jsonl(run / "metrics.jsonl") if "loss" in r]
    losses = [r["loss"] for r in sorted(recs, key=lambda r: r["step"])]
    n = min(reference_steps, len(losses))
    settings = PipelineSettings("ref", steps=n, batch_size=cfg.training.batch_size,
                                num_microbatches=cfg.training.num_microbatches)
    ref, _, _ = reference_step(cfg.model_spec_dict(), settings, seed=cfg.job.seed, optimizer=cfg.training.optimizer,
                               lr=cfg.training.learning_rate, steps=n)
    dev = max((abs(a - b) / max(abs(b), 1e-8) for a, b in zip(losses[:n], ref)), default=float("nan"))
    spec = cfg.build_model_spec()
    workers = {w["worker_id"]: w for w in (cluster_status or {}).get("workers", [])}
    hw = [f"{s['worker']} ({s['backend']}, {(workers.get(s['worker_id'], {}).get('device') or {}).get('name', '?')})"
          for s in plan["stages"]]
    stage_rows = []
    for s in plan["stages"]:
        st = summary["stages"].get(str(s["stage"]), {})
        stage_rows.append([s["stage"], s["worker"], s["backend"], f"{s['layers'][0]}-{s['layers'][1] - 1}",
                           f"{s['memory']['required'] / 1e9:.2f} / {s['memory']['budget'] / 1e9:.2f}",
                           f"{st.get('device_peak_bytes', 0) / 1e9:.2f}", f"{st.get('forward_s', 0) * 1e3:.1f}",
                           f"{st.get('backward_s', 0) * 1e3:.1f}", f"{st.get('comm_s', 0) * 1e3:.1f}",
                           f"{st.get('idle_s', 0) * 1e3:.1f}", f"{st.get('bytes_sent', 0) / 1e6:.2f}"])
    first, last = (summary["loss"][0][1], summary["loss"][-1][1]) if summary.get("loss") else (float("nan"),) * 2
    md = "\n\n".join([
        f"Run `{run.name}` on {' -> '.join(hw)}",
        f"Model: {cfg.model.type}, {spec.parameter_count() / 1e6:.1f}M params ({spec.num_layers} layers); batch "
        f"{cfg.training.batch_size}, {cfg.training.num_microbatches} microbatches, {cfg.training.optimizer}.",
        md_table(["steps", "loss first -> last", "ms/step", "MB/step",
                  f"max rel. loss deviation vs CPU single process (first {n} steps)"],
                 [[summary["steps"], f"{first:.4f} -> {last:.4f}", f"{(summary.get('mean_step_s') or 0) * 1e3:.1f}",
                   f"{summary.get('bytes_per_step', 0) / 1e6:.2f}", f"{dev:.2e}"]]),
        md_table(["stage", "worker", "backend", "layers", "planned GB (need / usable)", "device peak GB", "fwd ms",
                  "bwd ms", "comm ms", "idle ms", "MB sent/step"], stage_rows)])
    if write_doc:
        update_section(section, md)
    return md

"""Placement reports and prediction accuracy (reference planner/report.py:20-108)."""

from __future__ import annotations

GB = 1024 ** 3


def format_placement(plan, layer_names: list[str] | None = None, workers: dict | None = None) -> str:
    """``inspect placement``: per-stage memory breakdown and per-boundary transfer cost."""
    lines = [plan.format(layer_names), "", "Memory by stage:"]
    for s in plan.stages:
        unified = bool(workers and workers.get(s.worker_id, {}).get("unified_memory"))
        lines.append(s.memory.format(f"{s.worker_name} (stage {s.stage_index})", unified=unified))
    bds = plan.boundaries()
    if bds:
        lines += ["", "Boundaries (per microbatch):"]
        for b in bds:
            f = b["forward"]
            lines.append(f"  stage {b['from_stage']} -> {b['to_stage']}: {b['activation_bytes'] / 1e6:.2f} MB  "
                         f"[{f.get('kind', 'host')}] d2h {f.get('d2h_s', 0) * 1e3:.2f} ms + net "
                         f"{f.get('network_s', 0) * 1e3:.2f} ms + h2d {f.get('h2d_s', 0) * 1e3:.2f} ms")
    b = plan.bottleneck
    if b:
        lines += ["", f"Bottleneck: stage {b.stage_index} on {b.worker_name} "
                      f"({'compute' if b.compute_s >= b.comm_s else 'communication'}-bound)"]
    return "\n".join(lines)


def prediction_accuracy(plan_dict: dict, summary: dict) -> dict:
    """Planner prediction vs measured run (compute, memory, step time)."""
    out = {"stages": {}}
    for st in plan_dict.get("stages", []):
        idx = st["stage"]
        meas = summary.get("stages", {}).get(idx) or summary.get("stages", {}).get(str(idx)) or {}
        M = plan_dict.get("num_microbatches", 1)
        pred_compute = st["compute_s_per_mb"] * M
        actual_compute = meas.get("compute_s")
        pred_mem = st["memory"]["required"]
        actual_mem = meas.get("device_peak_bytes")
        row = {"predicted_compute_s": pred_compute, "actual_compute_s": actual_compute,
               "predicted_memory_bytes": pred_mem, "actual_peak_memory_bytes": actual_mem}
        if actual_compute:
            row["compute_error"] = (pred_compute - actual_compute) / actual_compute
        if actual_mem:
            row["memory_error"] = (pred_mem - actual_mem) / actual_mem
        out["stages"][idx] = row
    pred_step = plan_dict.get("predicted_step_s")
    actual_step = summary.get("mean_step_s")
    out["predicted_step_s"], out["actual_step_s"] = pred_step, actual_step
    if pred_step and actual_step:
        out["step_error"] = (pred_step - actual_step) / actual_step
    return out


def format_accuracy(acc: dict) -> str:
    lines = ["Prediction accuracy:"]
    if acc.get("actual_step_s"):
        lines.append(f"  step: predicted {acc['predicted_step_s'] * 1e3:.1f} ms, actual "
                     f"{acc['actual_step_s'] * 1e3:.1f} ms ({acc.get('step_error', 0):+.1%})")
    for idx, r in acc.get("stages", {}).items():
        parts = [f"  stage {idx}:"]
        if r.get("actual_compute_s"):
            parts.append(f"compute {r['predicted_compute_s'] * 1e3:.1f}/{r['actual_compute_s'] * 1e3:.1f} ms "
                         f"({r.get('compute_error', 0):+.1%})")
        if r.get("actual_peak_memory_bytes"):
            parts.append(f"memory {r['predicted_memory_bytes'] / GB:.2f}/{r['actual_peak_memory_bytes'] / GB:.2f} GB "
                         f"({r.get('memory_error', 0):+.1%})")
        lines.append(" ".join(parts))
    return "\n".join(lines)

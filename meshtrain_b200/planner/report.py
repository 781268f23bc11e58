"""Placement reports and prediction accuracy (reference planner/report.py:20-108)."""

from __future__ import annotations

GB = 1024 ** 3


_MEM_ROWS = ("parameters", "gradients", "master_weights", "optimizer_state", "optimizer_step_temporary",
             "saved_activations", "input_buffers", "output_buffers", "transport_buffers", "temporary_workspace")


def format_placement(plan, layer_names: list[str] | None = None, workers: dict | None = None) -> str:
    """``inspect placement``: stages, per-stage memory breakdown and per-boundary transfer cost.

    ``plan`` is a ``Plan`` or its ``to_dict()`` form (what the coordinator returns).
    """
    d = plan if isinstance(plan, dict) else plan.to_dict()
    gb = lambda n: f"{n / GB:8.2f} GB"  # noqa: E731
    lines = [f"Placement ({d['strategy']}), {'feasible' if d['feasible'] else 'NOT feasible'}", ""]
    for s in d["stages"]:
        a, b = s["layers"]
        names = f" ({layer_names[a]} .. {layer_names[b - 1]})" if layer_names else ""
        m = s["memory"]
        lines += [f"Stage {s['stage']} -> {s['worker']} [{s['backend']}]  layers {a}-{b - 1}{names}",
                  f"    compute {s['compute_s_per_mb'] * 1e3:.2f} ms/mb, send {s['comm_s_per_mb'] * 1e3:.2f} ms/mb"
                  f"{' (overlapped)' if s.get('overlap') else ''}"]
        unified = bool(workers and workers.get(s["worker_id"], {}).get("unified_memory"))
        lines.append(f"    {'total memory' + ('*' if unified else ''):<32}{gb(m['total'])}")
        lines.append(f"    {'usable':<32}{gb(m['usable'])}")
        lines += [f"    {k.replace('_', ' '):<32}{gb(m[k])}" for k in _MEM_ROWS if m.get(k)]
        lines.append(f"    {'required':<32}{gb(m['required'])}  ({'ok' if m['fits'] else 'OVER BUDGET'})")
        if m.get("host_offload"):
            lines.append(f"    {'offloaded to host DRAM':<32}{gb(m['host_offload'])}")
    if d.get("boundaries"):
        lines += ["", "Boundaries (per microbatch):"]
        for bd in d["boundaries"]:
            f = bd["forward"]
            lines.append(f"  Boundary {bd['from_stage']} -> {bd['to_stage']}: {bd['activation_bytes'] / 1e6:.2f} MB "
                         f"[{f.get('kind', 'host')}] d2h {f.get('d2h_s', 0) * 1e3:.2f} ms + link "
                         f"{f.get('network_s', 0) * 1e3:.2f} ms + h2d {f.get('h2d_s', 0) * 1e3:.2f} ms")
    if d["stages"]:
        b = max(d["stages"], key=lambda s: s["time_per_mb"])
        bound = "compute" if b["compute_s_per_mb"] >= b["comm_s_per_mb"] else "communication"
        lines += ["", f"Predicted: {d['predicted_step_s'] * 1e3:.1f} ms/step; bottleneck stage {b['stage']} on "
                      f"{b['worker']} ({bound}-bound)"]
    lines += [f"  excluded: {w} ({why})" for w, why in d.get("excluded", {}).items()]
    lines += [f"  VIOLATION: {v}" for v in d.get("violations", [])]
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

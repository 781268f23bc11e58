"""Aggregate STEP_COMPLETE records into a run summary (reference summary.py:9-80).

Only the last attempt counts and warm-up steps are excluded; per stage it
reports mean step/compute/comm/exposed/idle times, device-timed fields when
present (step_ms, bubble, exposed p2p), and stage 0's loss trajectory.
"""

from __future__ import annotations

from statistics import mean

_MEAN_KEYS = ("step_s", "forward_s", "backward_s", "optimizer_s", "compute_s", "comm_s", "overlapped_s",
              "exposed_communication_s", "idle_s", "overlap_ratio", "utilization", "device_step_ms",
              "bubble_fraction", "exposed_p2p_ms", "bytes_sent", "bytes_received")


def summarize(records: list[dict], warmup_steps: int = 1) -> dict:
    recs = [r for r in records if r.get("event", "STEP_COMPLETE") == "STEP_COMPLETE"]
    if not recs:
        return {"steps": 0, "stages": {}}
    last_attempt = max(r.get("attempt", 0) for r in recs)
    recs = [r for r in recs if r.get("attempt", 0) == last_attempt]
    steps = sorted({r["step"] for r in recs})
    timed = [s for s in steps if s >= steps[0] + warmup_steps] or steps
    stages: dict[int, dict] = {}
    for idx in sorted({r["stage"] for r in recs}):
        rs = [r for r in recs if r["stage"] == idx and r["step"] in timed]
        st = {"worker": rs[0].get("worker"), "backend": rs[0].get("backend"), "steps": len(rs)}
        for k in _MEAN_KEYS:
            vals = [r[k] for r in rs if isinstance(r.get(k), (int, float))]
            if vals:
                st[k] = mean(vals)
        peaks = [r.get("memory", {}).get("device_peak", 0) for r in rs]
        st["device_peak_bytes"] = max(peaks) if peaks else 0
        stages[idx] = st
    # the host runtime reports the loss on stage 0, the device engine on the last stage
    loss_stage = min((r["stage"] for r in recs if "loss" in r), default=min(stages))
    first = [r for r in recs if r["stage"] == loss_stage]
    losses = [(r["step"], r["loss"]) for r in sorted(first, key=lambda r: r["step"]) if "loss" in r]
    step_means = [st["step_s"] for st in stages.values() if "step_s" in st]
    out = {"steps": len(steps), "timed_steps": len(timed), "attempt": last_attempt, "stages": stages,
           "bytes_per_step": sum(st.get("bytes_sent", 0.0) for st in stages.values()),
           "mean_step_s": max(step_means) if step_means else None, "loss": losses,
           "final_loss": losses[-1][1] if losses else None}
    sps = [r.get("samples_per_s") for r in first if r["step"] in timed and r.get("samples_per_s")]
    if sps:
        out["samples_per_s"] = mean(sps)
    tps = [r.get("tokens_per_s") for r in first if r["step"] in timed and r.get("tokens_per_s")]
    if tps:
        out["tokens_per_s"] = mean(tps)
    return out


def format_summary(s: dict) -> str:
    if not s.get("steps"):
        return "no steps recorded"
    lines = [f"steps: {s['steps']} (timed {s['timed_steps']}, attempt {s['attempt']})"]
    if s.get("mean_step_s"):
        lines.append(f"mean step: {s['mean_step_s'] * 1e3:.1f} ms")
    if s.get("samples_per_s"):
        lines.append(f"throughput: {s['samples_per_s']:.1f} samples/s")
    if s.get("tokens_per_s"):
        lines.append(f"throughput: {s['tokens_per_s']:.0f} tokens/s")
    if s.get("final_loss") is not None:
        lines.append(f"final loss: {s['final_loss']:.4f}")
    for idx, st in s["stages"].items():
        extra = ""
        if "bubble_fraction" in st:
            extra = f" bubble={st['bubble_fraction']:.1%} exposed_p2p={st.get('exposed_p2p_ms', 0):.2f}ms"
        lines.append(f"  stage {idx} [{st.get('backend')}] {st.get('worker')}: step={st.get('step_s', 0) * 1e3:.1f}ms "
                     f"compute={st.get('compute_s', 0) * 1e3:.1f}ms comm={st.get('comm_s', 0) * 1e3:.1f}ms "
                     f"exposed={st.get('exposed_communication_s', 0) * 1e3:.1f}ms idle={st.get('idle_s', 0) * 1e3:.1f}ms"
                     + extra)
    return "\n".join(lines)

"""``meshtrain benchmark pipeline``: the four execution modes of the host runtime on one model.

    gpipe + blocking sends      gpipe + async sends
    1f1b  + blocking sends      1f1b  + async sends (pooled, pinned staging)

Locally every stage is a process on loopback TCP.  Loopback is far faster than
a LAN, so the links are throttled to ``bandwidth_mbps`` / ``latency_ms`` unless
``bandwidth_mbps`` is None, and each report names the link it used.  With a
cluster client each mode is a coordinator job instead.  Per mode: steps/s,
samples/s, step time, peak saved activations, idle / communication / exposed
communication per stage, overlap, bytes per step, the final loss, and whether
the loss trajectory equals the first mode's (the reference's V1 vs V1.5
comparison, experiments/pipeline_bench.py and docs/v1-vs-v1.5.md).
"""

from __future__ import annotations

import json
import time
from dataclasses import dataclass
from pathlib import Path

from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.summary import summarize
from meshtrain_b200.telemetry import new_run_id, read_jsonl
from meshtrain_b200.utils.trace_report import ascii_timeline, format_breakdown, write_run_timeline


@dataclass(frozen=True)
class Mode:
    label: str
    schedule: str
    async_sends: bool

    @property
    def slug(self) -> str:
        return f"{self.schedule}-{'async' if self.async_sends else 'blocking'}"


MODES = (Mode("gpipe + blocking", "gpipe", False), Mode("gpipe + async", "gpipe", True),
         Mode("1f1b + blocking", "1f1b", False), Mode("1f1b + async", "1f1b", True))
DEFAULT_MODEL = {"type": "tiny_transformer", "layers": 6, "hidden_size": 256, "heads": 4, "vocab_size": 512,
                 "seq_len": 64}
COLUMNS = ("mode", "steps/s", "samples/s", "step ms", "peak act MB (max)", "peak act MB (stage 0)",
           "saved mb (stage 0)", "idle ms", "comm ms", "exposed ms", "overlap", "MB/step", "final loss", "same loss")


def mode_row(label: str, summary: dict, records: list[dict], batch: int, losses: list[float],
             baseline: list[float] | None) -> dict:
    """One mode's figures from its run summary and STEP_COMPLETE records."""
    stages = summary["stages"]
    n = len(stages)
    step_s = summary["mean_step_s"]
    totals = {k: sum(v.get(k, 0.0) for v in stages.values())
              for k in ("comm_s", "idle_s", "exposed_communication_s", "overlapped_s", "bytes_sent")}
    peaks = {}
    for stage in stages:
        mem = [r["memory"] for r in records if r.get("stage") == stage and r.get("event", "STEP_COMPLETE") == "STEP_COMPLETE"]
        peaks[stage] = (max((m.get("saved_activations_peak", 0) for m in mem), default=0),
                        max((m.get("saved_microbatches_peak", 0) for m in mem), default=0))
    first = peaks[min(stages)]
    same = None if baseline is None else max(abs(a - b) / max(abs(b), 1e-9) for a, b in zip(losses, baseline)) < 1e-5
    return {"mode": label, "steps_per_s": 1 / step_s, "samples_per_s": batch / step_s, "step_ms": step_s * 1e3,
            "peak_act_MB_max": max(p[0] for p in peaks.values()) / 1e6, "peak_act_MB_stage0": first[0] / 1e6,
            "peak_saved_mb_stage0": first[1], "idle_ms": totals["idle_s"] / n * 1e3,
            "comm_ms": totals["comm_s"] / n * 1e3, "exposed_ms": totals["exposed_communication_s"] / n * 1e3,
            "overlap_ratio": totals["overlapped_s"] / totals["comm_s"] if totals["comm_s"] else 0.0,
            "MB_per_step": totals["bytes_sent"] / 1e6, "final_loss": losses[-1], "loss_matches_first": same}


def _cells(r: dict) -> list:
    same = "-" if r["loss_matches_first"] is None else ("yes" if r["loss_matches_first"] else "NO")
    return [r["mode"], f"{r['steps_per_s']:.2f}", f"{r['samples_per_s']:.1f}", f"{r['step_ms']:.0f}",
            f"{r['peak_act_MB_max']:.1f}", f"{r['peak_act_MB_stage0']:.1f}", r["peak_saved_mb_stage0"],
            f"{r['idle_ms']:.0f}", f"{r['comm_ms']:.0f}", f"{r['exposed_ms']:.0f}", f"{r['overlap_ratio']:.0%}",
            f"{r['MB_per_step']:.2f}", f"{r['final_loss']:.4f}", same]


def run_local_benchmark(model_cfg: dict | None = None, num_stages: int = 3, batch_size: int = 32,
                        num_microbatches: int = 8, steps: int = 8, bandwidth_mbps: float | None = 100.0,
                        latency_ms: float = 1.0, runs_dir: str = "runs", write_doc: bool = True,
                        devices: list[str] | None = None, compression: str | None = None) -> dict:
    """Runs the four modes locally; ``compression`` ("bf16" / "fp16") sends fp32 boundary tensors as
    16-bit floats (the "same loss" column then compares against the first mode, also compressed)."""
    model_cfg = model_cfg or DEFAULT_MODEL
    spec = build_model_spec(model_cfg)
    n = spec.num_layers
    devices = devices or ["cpu"] * num_stages
    stages = [LocalStage((n * i // num_stages, n * (i + 1) // num_stages), devices[i]) for i in range(num_stages)]
    link = (bandwidth_mbps * 1e6 / 8, latency_ms / 1e3) if bandwidth_mbps else None
    run_id = new_run_id("pipeline-bench")
    run_dir = Path(runs_dir) / run_id
    rows, baseline, last = [], None, None
    for mode in MODES:
        settings = PipelineSettings(f"bench-{mode.slug}", steps=steps, batch_size=batch_size,
                                    num_microbatches=num_microbatches, schedule=mode.schedule,
                                    async_transport=mode.async_sends, log_every=10 ** 6,
                                    wire_compression=compression)
        results = run_local_pipeline(model_cfg, stages, settings, optimizer="adamw", lr=3e-4, transport="tcp",
                                     link_emulation=link)
        records = [m for r in results for m in r.step_metrics]
        summary = summarize(records, warmup_steps=min(2, steps - 1))
        rows.append(mode_row(mode.label, summary, records, batch_size, results[0].losses, baseline))
        baseline = baseline or results[0].losses
        lanes = [(r.stage_index, r.worker, r.timeline or []) for r in results]
        write_run_timeline(run_dir / f"timeline-{mode.slug}.json", lanes)
        last = (summary, lanes)
    meta = {"model": model_cfg, "parameters": spec.parameter_count(), "stages": [list(s.layers) for s in stages],
            "devices": devices, "batch_size": batch_size, "microbatches": num_microbatches, "steps": steps,
            "link": "loopback TCP (not emulated)" if link is None else
            f"emulated {bandwidth_mbps:g} Mbit/s, {latency_ms:g} ms per message, each direction",
            "compression": compression or "none"}
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "benchmark.json").write_text(json.dumps({"meta": meta, "rows": rows}, indent=2))
    breakdown, gantt = format_breakdown(last[0]), ascii_timeline(last[1], step=steps - 1)
    (run_dir / "timeline_report.txt").write_text(f"{breakdown}\n\n{gantt}\n")
    md = render_markdown(meta, rows, breakdown, gantt, run_id)
    if write_doc:
        update_section("pipeline-benchmark-local", md)
    return {"run_dir": str(run_dir), "meta": meta, "rows": rows, "markdown": md}


def render_markdown(meta: dict, rows: list[dict], breakdown: str, gantt: str, run_id: str) -> str:
    slow, fast = rows[0], rows[-1]
    return "\n\n".join([
        environment_line(),
        f"Run `{run_id}`. Model: {meta['model']['type']} ({meta['parameters'] / 1e6:.2f}M params), stages "
        f"{meta['stages']} on {', '.join(meta['devices'])}, batch {meta['batch_size']} = {meta['microbatches']} "
        f"microbatches, {meta['steps']} steps. Link: **{meta['link']}**"
        + (f", boundary tensors sent as {meta['compression']}." if meta.get("compression", "none") != "none" else "."),
        md_table(list(COLUMNS), [_cells(r) for r in rows]),
        f"**{slow['mode']} -> {fast['mode']}:** {slow['step_ms']:.0f} -> {fast['step_ms']:.0f} ms/step "
        f"({slow['step_ms'] / fast['step_ms']:.2f}x); exposed communication {slow['exposed_ms']:.0f} -> "
        f"{fast['exposed_ms']:.0f} ms/stage/step; stage-0 peak saved activations {slow['peak_act_MB_stage0']:.1f} -> "
        f"{fast['peak_act_MB_stage0']:.1f} MB.",
        f"Per-worker breakdown (last mode):\n\n```\n{breakdown}\n```",
        f"Last step of the last mode:\n\n```\n{gantt}\n```"])


def run_cluster_benchmark(client, config_raw: dict, poll_s: float = 1.0, write_doc: bool = True) -> dict:
    rows, baseline = [], None
    batch = config_raw["training"]["batch_size"]
    for mode in MODES:
        cfg = json.loads(json.dumps(config_raw))  # a deep copy per mode
        cfg.setdefault("job", {})["name"] = f"bench-{mode.slug}"
        cfg.setdefault("pipeline", {})["schedule"] = mode.schedule
        cfg.setdefault("transport", {})["async"] = mode.async_sends
        job_id = client.start_job(cfg)["job_id"]
        while (job := client.job(job_id))["status"] == "RUNNING":
            time.sleep(poll_s)
        if job["status"] != "COMPLETED" or not job.get("summary"):
            rows.append({"mode": mode.label, "error": job.get("error")})
            continue
        losses = [loss for _step, loss in sorted(job["losses"])]
        summary = dict(job["summary"], stages={int(k): v for k, v in job["summary"]["stages"].items()})
        records = read_jsonl(Path(job["run_dir"]) / "metrics.jsonl")
        rows.append(dict(mode_row(mode.label, summary, records, batch, losses, baseline), job=job["job_id"]))
        baseline = baseline or losses
    good = [r for r in rows if "error" not in r]
    table = md_table(["mode", "job", "steps/s", "step ms", "peak act MB (stage 0)", "exposed ms", "overlap", "MB/step",
                      "final loss"],
                     [[r["mode"], r["job"], f"{r['steps_per_s']:.2f}", f"{r['step_ms']:.0f}",
                       f"{r['peak_act_MB_stage0']:.1f}", f"{r['exposed_ms']:.0f}", f"{r['overlap_ratio']:.0%}",
                       f"{r['MB_per_step']:.2f}", f"{r['final_loss']:.4f}"] for r in good])
    md = "\n\n".join([environment_line(), "Cluster run (real devices and network) through the coordinator.", table]
                     + [f"- {r['mode']}: FAILED {r['error']}" for r in rows if "error" in r])
    if write_doc:
        update_section("pipeline-benchmark-cluster", md)
    return {"rows": rows, "markdown": md}

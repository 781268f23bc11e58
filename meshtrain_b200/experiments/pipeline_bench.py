"""``meshtrain benchmark pipeline``: the four execution modes on one model (reference
experiments/pipeline_bench.py:1-170).

    gpipe + blocking sends      gpipe + async sends
    1f1b  + blocking sends      1f1b  + async sends (+ buffer reuse, pinned staging)

Locally every stage is its own process over loopback TCP; because loopback is
far faster than a LAN, links are emulated (bandwidth + latency throttle) unless
``bandwidth_mbps`` is None, and every report names the link used.  With a
cluster client the modes are submitted as jobs instead.  Per mode: steps/s,
samples/s, step time, peak saved activations, idle / communication / exposed
communication, overlap, bytes per step, loss, and whether the loss trajectory
equals the first mode's.
"""

from __future__ import annotations

import json
import time
from pathlib import Path

from meshtrain_b200.experiments.results_doc import environment_line, md_table, update_section
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.local import LocalStage, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings
from meshtrain_b200.summary import summarize
from meshtrain_b200.telemetry import new_run_id
from meshtrain_b200.utils.trace_report import ascii_timeline, format_breakdown, write_run_timeline

MODES = [("gpipe + blocking", "gpipe", False), ("gpipe + async", "gpipe", True),
         ("1f1b + blocking", "1f1b", False), ("1f1b + async", "1f1b", True)]
DEFAULT_MODEL = {"type": "tiny_transformer", "layers": 6, "hidden_size": 256, "heads": 4, "vocab_size": 512,
                 "seq_len": 64}


def _peak_act(records: list[dict], stage: int) -> tuple[int, int]:
    rs = [r for r in records if r.get("stage") == stage and r.get("event", "STEP_COMPLETE") == "STEP_COMPLETE"]
    return (max((r["memory"].get("saved_activations_peak", 0) for r in rs), default=0),
            max((r["memory"].get("saved_microbatches_peak", 0) for r in rs), default=0))


def _row(name: str, s: dict, records: list[dict], batch: int, losses: list[float], ref: list[float] | None) -> dict:
    st = s["stages"]
    step = s["mean_step_s"]

    def total(k):
        return sum(v.get(k, 0.0) for v in st.values())

    comm = total("comm_s")
    acts = {i: _peak_act(records, i) for i in st}
    first = min(st)
    return {"mode": name, "steps_per_s": 1 / step, "samples_per_s": batch / step, "step_ms": step * 1e3,
            "peak_act_MB_max": max(a for a, _ in acts.values()) / 1e6, "peak_act_MB_stage0": acts[first][0] / 1e6,
            "peak_saved_mb_stage0": acts[first][1], "idle_ms": total("idle_s") / len(st) * 1e3,
            "comm_ms": comm / len(st) * 1e3, "exposed_ms": total("exposed_communication_s") / len(st) * 1e3,
            "overlap_ratio": total("overlapped_s") / comm if comm else 0.0,
            "MB_per_step": total("bytes_sent") / 1e6, "final_loss": losses[-1],
            "loss_matches_first": None if ref is None else
            max(abs(a - b) / max(abs(b), 1e-9) for a, b in zip(losses, ref)) < 1e-5}


def run_local_benchmark(model_cfg: dict | None = None, num_stages: int = 3, batch_size: int = 32,
                        num_microbatches: int = 8, steps: int = 8, bandwidth_mbps: float | None = 100.0,
                        latency_ms: float = 1.0, runs_dir: str = "runs", write_doc: bool = True,
                        devices: list[str] | None = None) -> dict:
    model_cfg = model_cfg or DEFAULT_MODEL
    n = build_model_spec(model_cfg).num_layers
    devices = devices or ["cpu"] * num_stages
    stages = [LocalStage((n * i // num_stages, n * (i + 1) // num_stages), devices[i]) for i in range(num_stages)]
    link = (bandwidth_mbps * 1e6 / 8, latency_ms / 1e3) if bandwidth_mbps else None
    run_id = new_run_id("pipeline-bench")
    run_dir = Path(runs_dir) / run_id
    rows, ref, last = [], None, None
    for name, schedule, asyn in MODES:
        settings = PipelineSettings(f"bench-{schedule}-{int(asyn)}", steps=steps, batch_size=batch_size,
                                    num_microbatches=num_microbatches, schedule=schedule, async_transport=asyn,
                                    log_every=10 ** 6)
        res = run_local_pipeline(model_cfg, stages, settings, optimizer="adamw", lr=3e-4, transport="tcp",
                                 link_emulation=link)
        records = [m for r in res for m in r.step_metrics]
        s = summarize(records, warmup_steps=min(2, steps - 1))
        rows.append(_row(name, s, records, batch_size, res[0].losses, ref))
        ref = ref or res[0].losses
        lanes = [(r.stage_index, r.worker, r.timeline or []) for r in res]
        write_run_timeline(run_dir / f"timeline-{schedule}-{'async' if asyn else 'blocking'}.json", lanes)
        last = (s, lanes)
    spec = build_model_spec(model_cfg)
    meta = {"model": model_cfg, "parameters": spec.parameter_count(), "stages": [list(s.layers) for s in stages],
            "devices": devices, "batch_size": batch_size, "microbatches": num_microbatches, "steps": steps,
            "link": "loopback TCP (not emulated)" if link is None else
            f"emulated {bandwidth_mbps:g} Mbit/s, {latency_ms:g} ms per message, each direction"}
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "benchmark.json").write_text(json.dumps({"meta": meta, "rows": rows}, indent=2))
    breakdown, gantt = format_breakdown(last[0]), ascii_timeline(last[1], step=steps - 1)
    (run_dir / "timeline_report.txt").write_text(breakdown + "\n\n" + gantt + "\n")
    md = render_markdown(meta, rows, breakdown, gantt, run_id)
    if write_doc:
        update_section("pipeline-benchmark-local", md)
    return {"run_dir": str(run_dir), "meta": meta, "rows": rows, "markdown": md}


def render_markdown(meta: dict, rows: list[dict], breakdown: str, gantt: str, run_id: str) -> str:
    a, b = rows[0], rows[-1]
    table = md_table(["mode", "steps/s", "samples/s", "step ms", "peak act MB (max)", "peak act MB (stage 0)",
                      "saved mb (stage 0)", "idle ms", "comm ms", "exposed ms", "overlap", "MB/step", "final loss",
                      "same loss"],
                     [[r["mode"], f"{r['steps_per_s']:.2f}", f"{r['samples_per_s']:.1f}", f"{r['step_ms']:.0f}",
                       f"{r['peak_act_MB_max']:.1f}", f"{r['peak_act_MB_stage0']:.1f}", r["peak_saved_mb_stage0"],
                       f"{r['idle_ms']:.0f}", f"{r['comm_ms']:.0f}", f"{r['exposed_ms']:.0f}",
                       f"{r['overlap_ratio']:.0%}", f"{r['MB_per_step']:.2f}", f"{r['final_loss']:.4f}",
                       "-" if r["loss_matches_first"] is None else ("yes" if r["loss_matches_first"] else "NO")]
                      for r in rows])
    return "\n\n".join([
        environment_line(),
        f"Run `{run_id}`. Model: {meta['model']['type']} ({meta['parameters'] / 1e6:.2f}M params), stages "
        f"{meta['stages']} on {', '.join(meta['devices'])}, batch {meta['batch_size']} = {meta['microbatches']} "
        f"microbatches, {meta['steps']} steps. Link: **{meta['link']}**.",
        table,
        f"**{a['mode']} -> {b['mode']}:** {a['step_ms']:.0f} -> {b['step_ms']:.0f} ms/step "
        f"({a['step_ms'] / b['step_ms']:.2f}x); exposed communication {a['exposed_ms']:.0f} -> {b['exposed_ms']:.0f} "
        f"ms/stage/step; stage-0 peak saved activations {a['peak_act_MB_stage0']:.1f} -> "
        f"{b['peak_act_MB_stage0']:.1f} MB.",
        "Per-worker breakdown (last mode):\n\n```\n" + breakdown + "\n```",
        "Last step of the last mode:\n\n```\n" + gantt + "\n```"])


def run_cluster_benchmark(client, config_raw: dict, poll_s: float = 1.0, write_doc: bool = True) -> dict:
    rows, ref = [], None
    batch = config_raw["training"]["batch_size"]
    for name, schedule, asyn in MODES:
        cfg = json.loads(json.dumps(config_raw))
        cfg.setdefault("job", {})["name"] = f"bench-{schedule}-{'async' if asyn else 'blocking'}"
        cfg.setdefault("pipeline", {})["schedule"] = schedule
        cfg.setdefault("transport", {})["async"] = asyn
        job = client.start_job(cfg)
        while (j := client.job(job["job_id"]))["status"] == "RUNNING":
            time.sleep(poll_s)
        if j["status"] != "COMPLETED" or not j.get("summary"):
            rows.append({"mode": name, "error": j.get("error")})
            continue
        losses = [loss for _, loss in sorted(j["losses"])]
        s = j["summary"]
        s["stages"] = {int(k): v for k, v in s["stages"].items()}
        from meshtrain_b200.telemetry import read_jsonl

        records = read_jsonl(Path(j["run_dir"]) / "metrics.jsonl")
        rows.append({**_row(name, s, records, batch, losses, ref), "job": j["job_id"]})
        ref = ref or losses
    ok = [r for r in rows if "error" not in r]
    md = "\n\n".join([environment_line(), "Cluster run (real devices and network) through the coordinator.",
                      md_table(["mode", "job", "steps/s", "step ms", "peak act MB (stage 0)", "exposed ms", "overlap",
                                "MB/step", "final loss"],
                               [[r["mode"], r["job"], f"{r['steps_per_s']:.2f}", f"{r['step_ms']:.0f}",
                                 f"{r['peak_act_MB_stage0']:.1f}", f"{r['exposed_ms']:.0f}", f"{r['overlap_ratio']:.0%}",
                                 f"{r['MB_per_step']:.2f}", f"{r['final_loss']:.4f}"] for r in ok])]
                     + [f"- {r['mode']}: FAILED {r['error']}" for r in rows if "error" in r])
    if write_doc:
        update_section("pipeline-benchmark-cluster", md)
    return {"rows": rows, "markdown": md}

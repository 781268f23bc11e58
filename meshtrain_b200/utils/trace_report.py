"""Run-level timeline artefacts: merged Chrome trace, per-worker breakdown, ASCII Gantt.

(reference runtime/trace_report.py:21-77)
"""

from __future__ import annotations

from pathlib import Path

from meshtrain_b200.utils.timeline import COMM_WORK, COMPUTE, chrome_events_from_export, write_chrome_trace

MAX_SPANS_PER_STAGE = 50_000


def write_run_timeline(path, stages: list[tuple[int, str, list[dict]]]) -> Path:
    """``stages``: (stage index, worker, exported spans) -> one Chrome trace file."""
    return write_chrome_trace(path, [chrome_events_from_export(sp[-MAX_SPANS_PER_STAGE:], idx, w)
                                     for idx, w, sp in stages])


def worker_breakdown(summary: dict) -> dict:
    out = {}
    step = summary.get("mean_step_s") or 0.0
    if not step:
        return out
    for idx, st in summary.get("stages", {}).items():
        comm = st.get("comm_s", 0.0)
        out[idx] = {"worker": st.get("worker"), "backend": st.get("backend"),
                    "compute": st.get("compute_s", 0.0) / step, "communication": comm / step,
                    "exposed_communication": st.get("exposed_communication_s", comm) / step,
                    "idle": st.get("idle_s", 0.0) / step, "overlap_ratio": st.get("overlap_ratio", 0.0)}
    return out


def format_breakdown(summary: dict) -> str:
    lines = []
    for idx, b in worker_breakdown(summary).items():
        lines += [f"Worker {b['worker']} (stage {idx}, {b['backend']})", "",
                  f"  compute               {b['compute']:6.0%}",
                  f"  communication         {b['communication']:6.0%}   (overlap ratio {b['overlap_ratio']:.0%})",
                  f"  exposed communication {b['exposed_communication']:6.0%}",
                  f"  idle                  {b['idle']:6.0%}", ""]
    return "\n".join(lines).rstrip()


_GLYPH = {"FORWARD_COMPUTE": "F", "BACKWARD_COMPUTE": "B", "OPTIMIZER_STEP": "O", "NETWORK_SEND": ">",
          "NETWORK_RECV": "<", "P2P_SEND": ">", "P2P_RECV": "<", "D2H_COPY": "d", "H2D_COPY": "h",
          "SERIALIZE": "s", "DESERIALIZE": "s"}


def ascii_timeline(stages: list[tuple[int, str, list[dict]]], step: int, width: int = 96) -> str:
    """One step as text: a compute lane and a transfer lane per stage."""
    spans = [s for _, _, ss in stages for s in ss if s.get("step") == step]
    if not spans:
        return f"(no spans for step {step})"
    t0 = min(s["start"] for s in spans)
    t1 = max(s["end"] for s in spans)
    scale = (width - 1) / max(t1 - t0, 1e-9)
    lines = [f"step {step}: {(t1 - t0) * 1000:.1f} ms   F forward  B backward  O optimizer  "
             "> send  < recv  d/h device copies  . idle"]
    for idx, _w, ss in stages:
        for lane, cats in (("compute ", COMPUTE), ("transfer", COMM_WORK)):
            row = ["."] * width
            for s in ss:
                if s.get("step") != step or s["category"] not in cats:
                    continue
                a, b = int((s["start"] - t0) * scale), int((s["end"] - t0) * scale)
                for i in range(a, max(b, a + 1)):
                    if 0 <= i < width:
                        row[i] = _GLYPH.get(s["category"], "#")
            lines.append(f"stage {idx} {lane} |{''.join(row)}|")
    return "\n".join(lines)

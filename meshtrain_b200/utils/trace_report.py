"""Run-level views of the stages' timelines.

* ``write_run_timeline``: every stage's spans in one Chrome trace file (one
  process row per stage), capped per stage so a long run stays loadable.
* ``format_breakdown``: each worker's step time split into compute,
  communication (and how much of it overlapped), exposed communication and
  idle, from a run summary.
* ``ascii_timeline``: one step drawn as text, a compute lane and a transfer
  lane per stage, for terminals and ``timeline_report.txt``.

Same artefacts as the reference's report (runtime/trace_report.py:21-77).
"""

from __future__ import annotations

from pathlib import Path

from meshtrain_b200.utils.timeline import COMM_WORK, COMPUTE, chrome_events_from_export, write_chrome_trace

MAX_SPANS_PER_STAGE = 50_000

# one character per span category in the text timeline
LANE_CHARS = {
    "FORWARD_COMPUTE": "F", "BACKWARD_COMPUTE": "B", "OPTIMIZER_STEP": "O",
    "NETWORK_SEND": ">", "P2P_SEND": ">", "NETWORK_RECV": "<", "P2P_RECV": "<",
    "D2H_COPY": "d", "H2D_COPY": "h", "SERIALIZE": "s", "DESERIALIZE": "s",
}
LEGEND = "F forward  B backward  O optimizer  > send  < recv  d/h device copies  . idle"


def write_run_timeline(path, stages: list[tuple[int, str, list[dict]]]) -> Path:
    """``stages``: (stage index, worker, exported spans) -> one Chrome trace file."""
    per_stage = [chrome_events_from_export(spans[-MAX_SPANS_PER_STAGE:], index, worker)
                 for index, worker, spans in stages]
    return write_chrome_trace(path, per_stage)


def worker_breakdown(summary: dict) -> dict:
    """Per stage: fractions of the mean step spent in each activity."""
    step_s = summary.get("mean_step_s") or 0.0
    if step_s <= 0:
        return {}
    shares = {}
    for index, st in summary.get("stages", {}).items():
        comm = st.get("comm_s", 0.0)
        shares[index] = {
            "worker": st.get("worker"), "backend": st.get("backend"),
            "compute": st.get("compute_s", 0.0) / step_s,
            "communication": comm / step_s,
            "exposed_communication": st.get("exposed_communication_s", comm) / step_s,
            "idle": st.get("idle_s", 0.0) / step_s,
            "overlap_ratio": st.get("overlap_ratio", 0.0),
        }
    return shares


def format_breakdown(summary: dict) -> str:
    blocks = []
    for index, b in worker_breakdown(summary).items():
        rows = [("compute", b["compute"], ""),
                ("communication", b["communication"], f"   (overlap ratio {b['overlap_ratio']:.0%})"),
                ("exposed communication", b["exposed_communication"], ""),
                ("idle", b["idle"], "")]
        body = "\n".join(f"  {name:<21} {share:6.0%}{note}" for name, share, note in rows)
        blocks.append(f"Worker {b['worker']} (stage {index}, {b['backend']})\n\n{body}")
    return "\n\n".join(blocks)


def _lane(spans: list[dict], categories, t0: float, scale: float, width: int) -> str:
    cells = ["."] * width
    for span in spans:
        if span["category"] not in categories:
            continue
        first = int((span["start"] - t0) * scale)
        last = max(int((span["end"] - t0) * scale), first + 1)
        char = LANE_CHARS.get(span["category"], "#")
        for i in range(max(first, 0), min(last, width)):
            cells[i] = char
    return "".join(cells)


def ascii_timeline(stages: list[tuple[int, str, list[dict]]], step: int, width: int = 96) -> str:
    """One step as text: a compute lane and a transfer lane per stage."""
    of_step = {index: [s for s in spans if s.get("step") == step] for index, _w, spans in stages}
    everything = [s for spans in of_step.values() for s in spans]
    if not everything:
        return f"(no spans for step {step})"
    t0 = min(s["start"] for s in everything)
    t1 = max(s["end"] for s in everything)
    scale = (width - 1) / max(t1 - t0, 1e-9)
    out = [f"step {step}: {(t1 - t0) * 1000:.1f} ms   {LEGEND}"]
    for index, _w, _spans in stages:
        for label, categories in (("compute ", COMPUTE), ("transfer", COMM_WORK)):
            out.append(f"stage {index} {label} |{_lane(of_step[index], categories, t0, scale, width)}|")
    return "\n".join(out)

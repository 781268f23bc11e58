"""Per-stage execution timeline and interval-derived step metrics.

Spans are ``[start, end)`` wall-clock intervals with a category.  Step metrics
come from interval arithmetic, so overlap is measured, not assumed
(reference runtime/timeline.py:30-181):

    compute        = |U compute spans|          communication = |U transfer spans|
    overlapped     = |compute n communication|  exposed       = communication - overlapped
    idle           = step wall - |compute U communication|

GPU stages additionally record device-timed spans from CUDA events
(``add_device_spans``); those carry the same categories so one Chrome trace
shows both.
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass
from pathlib import Path

COMPUTE = ("FORWARD_COMPUTE", "BACKWARD_COMPUTE", "OPTIMIZER_STEP")
TRANSFER = ("D2H_COPY", "SERIALIZE", "QUEUE_WAIT", "NETWORK_SEND", "NETWORK_RECV", "DESERIALIZE", "H2D_COPY",
            "P2P_SEND", "P2P_RECV")
WAIT = ("WAIT_FORWARD", "WAIT_BACKWARD", "WAIT_SEND")
# QUEUE_WAIT is latency (a message waiting in the outbound queue), not transfer work.
COMM_WORK = tuple(c for c in TRANSFER if c != "QUEUE_WAIT")


@dataclass
class Span:
    category: str
    start: float
    end: float
    thread: str
    step: int | None = None
    microbatch: int | None = None
    args: dict | None = None

    @property
    def duration(self) -> float:
        return max(0.0, self.end - self.start)


def union(iv):
    merged: list[list[float]] = []
    for a, b in sorted(x for x in iv if x[1] > x[0]):
        if merged and a <= merged[-1][1]:
            merged[-1][1] = max(merged[-1][1], b)
        else:
            merged.append([a, b])
    return [(a, b) for a, b in merged]


def intersect(x, y):
    out, i, j = [], 0, 0
    while i < len(x) and j < len(y):
        a, b = max(x[i][0], y[j][0]), min(x[i][1], y[j][1])
        if a < b:
            out.append((a, b))
        if x[i][1] < y[j][1]:
            i += 1
        else:
            j += 1
    return out


def length(iv) -> float:
    return sum(b - a for a, b in iv)


class Timeline:
    def __init__(self, worker: str = "local", stage: int = 0, enabled: bool = True):
        self.worker, self.stage, self.enabled = worker, stage, enabled
        self._wall0 = time.time()
        self._perf0 = time.perf_counter()
        self._spans: list[Span] = []
        self._lock = threading.Lock()

    def now(self) -> float:
        return self._wall0 + (time.perf_counter() - self._perf0)

    def add(self, category: str, start: float, end: float, step=None, microbatch=None, **args) -> None:
        if not self.enabled:
            return
        sp = Span(category, start, end, threading.current_thread().name, step, microbatch, args or None)
        with self._lock:
            self._spans.append(sp)

    class _Scope:
        def __init__(self, tl, category, step, microbatch, args):
            self.tl, self.category, self.step, self.mb, self.args = tl, category, step, microbatch, args

        def __enter__(self):
            self.t0 = self.tl.now()
            return self

        def __exit__(self, *exc):
            self.tl.add(self.category, self.t0, self.tl.now(), self.step, self.mb, **self.args)
            return False

    def span(self, category: str, step=None, microbatch=None, **args):
        return Timeline._Scope(self, category, step, microbatch, args)

    def add_device_spans(self, spans: list[dict], step: int, step_start_wall: float, thread: str = "gpu") -> None:
        """Add CUDA-event spans (ms offsets from the step start) as wall-clock spans."""
        for s in spans:
            a = step_start_wall + s["start_ms"] / 1e3
            b = step_start_wall + s["end_ms"] / 1e3
            with self._lock:
                self._spans.append(Span(s["cat"], a, b, thread, step, s.get("mb"), {"device": True}))

    def spans(self, step: int | None = None) -> list[Span]:
        with self._lock:
            return [s for s in self._spans if step is None or s.step == step]

    def drop_before(self, t: float) -> None:
        with self._lock:
            self._spans = [s for s in self._spans if s.end >= t]

    def step_metrics(self, step: int, window: tuple[float, float]) -> dict:
        lo, hi = window
        inside = [s for s in self.spans() if s.end > lo and s.start < hi]

        def clipped(cats):
            return [(max(s.start, lo), min(s.end, hi)) for s in inside if s.category in cats]

        comp = union(clipped(COMPUTE))
        comm = union(clipped(COMM_WORK))
        busy = union(comp + comm)
        comp_s, comm_s = length(comp), length(comm)
        over = length(intersect(comp, comm))
        phases: dict[str, float] = {}
        for s in inside:
            if s.step == step or s.category in COMPUTE + COMM_WORK:
                phases[s.category] = phases.get(s.category, 0.0) + (min(s.end, hi) - max(s.start, lo))
        return {"compute_s": comp_s, "communication_s": comm_s, "overlapped_s": over,
                "exposed_communication_s": comm_s - over, "idle_s": max(0.0, (hi - lo) - length(busy)),
                "overlap_ratio": over / comm_s if comm_s > 0 else 0.0, "phase_s": phases}

    def to_chrome_events(self, pid: int | None = None) -> list[dict]:
        pid = self.stage if pid is None else pid
        tids: dict[str, int] = {}
        events = [{"ph": "M", "name": "process_name", "pid": pid,
                   "args": {"name": f"stage {self.stage} · {self.worker}"}}]
        for s in self.spans():
            tid = tids.setdefault(s.thread, len(tids))
            name = s.category if s.microbatch is None else f"{s.category} mb{s.microbatch}"
            events.append({"name": name, "cat": s.category, "ph": "X", "pid": pid, "tid": tid, "ts": s.start * 1e6,
                           "dur": s.duration * 1e6,
                           "args": {"step": s.step, "microbatch": s.microbatch, **(s.args or {})}})
        for thread, tid in tids.items():
            events.append({"ph": "M", "name": "thread_name", "pid": pid, "tid": tid, "args": {"name": thread}})
        return events

    def export(self) -> list[dict]:
        return [{"category": s.category, "start": s.start, "end": s.end, "thread": s.thread, "step": s.step,
                 "microbatch": s.microbatch, "args": s.args} for s in self.spans()]


def write_chrome_trace(path, stage_events: list[list[dict]]) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"traceEvents": [e for evs in stage_events for e in evs], "displayTimeUnit": "ms"}))
    return path


def chrome_events_from_export(spans: list[dict], stage: int, worker: str) -> list[dict]:
    tl = Timeline(worker, stage)
    tl._spans = [Span(s["category"], s["start"], s["end"], s.get("thread", "main"), s.get("step"),
                      s.get("microbatch"), s.get("args")) for s in spans]
    return tl.to_chrome_events()

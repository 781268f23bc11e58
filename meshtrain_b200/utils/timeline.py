"""Per-stage execution timeline and interval-derived step metrics.

Each record is a ``[start, end)`` wall-clock interval with a category.  The step
metrics the reference reports (runtime/timeline.py:30-181) are computed here by
one sweep over the interval end points: between two consecutive end points the
set of active category groups is constant, so the length of every combination
(compute only, communication only, both, neither) falls out of a single pass:

    compute        = time with compute active      communication = time with transfer work active
    overlapped     = time with both active         exposed       = communication - overlapped
    idle           = window - time with either active

GPU stages also record device-timed spans from CUDA events (``add_device_spans``)
under the same categories, so one Chrome trace shows host and device work.
"""

from __future__ import annotations

import json
import threading
import time
from collections import defaultdict
from pathlib import Path
from typing import NamedTuple

COMPUTE = ("FORWARD_COMPUTE", "BACKWARD_COMPUTE", "OPTIMIZER_STEP")
TRANSFER = ("D2H_COPY", "SERIALIZE", "QUEUE_WAIT", "NETWORK_SEND", "NETWORK_RECV", "DESERIALIZE", "H2D_COPY",
            "P2P_SEND", "P2P_RECV")
WAIT = ("WAIT_FORWARD", "WAIT_BACKWARD", "WAIT_SEND")
# A letter sitting in the outbound queue is latency, not transfer work, so QUEUE_WAIT
# counts toward neither communication nor overlap.
COMM_WORK = tuple(c for c in TRANSFER if c != "QUEUE_WAIT")

_GROUP = {**{c: "compute" for c in COMPUTE}, **{c: "comm" for c in COMM_WORK}}


class Span(NamedTuple):
    category: str
    start: float
    end: float
    thread: str = "main"
    step: int | None = None
    microbatch: int | None = None
    args: dict | None = None

    @property
    def duration(self) -> float:
        return self.end - self.start if self.end > self.start else 0.0

    def as_dict(self) -> dict:
        return dict(self._asdict())


def sweep(intervals: list[tuple[float, float, str]]) -> dict[frozenset, float]:
    """Length of time for which each combination of labels is active.

    ``intervals`` holds ``(start, end, label)``; the result maps a frozenset of
    labels active together to the total time they were (the empty set is not
    reported).  Empty or inverted intervals contribute nothing.
    """
    points: list[tuple[float, int, str]] = []
    for a, b, label in intervals:
        if b > a:
            points.append((a, 1, label))
            points.append((b, -1, label))
    points.sort(key=lambda p: (p[0], p[1]))
    active: dict[str, int] = defaultdict(int)
    out: dict[frozenset, float] = defaultdict(float)
    prev = None
    for t, delta, label in points:
        if prev is not None and t > prev:
            live = frozenset(k for k, n in active.items() if n > 0)
            if live:
                out[live] += t - prev
        active[label] += delta
        prev = t
    return dict(out)


def covered(intervals) -> float:
    """Total length covered by a collection of ``(start, end)`` intervals."""
    return sum(sweep([(a, b, "x") for a, b in intervals]).values())


def chrome_events(spans, pid: int, process_label: str) -> list[dict]:
    """Chrome-trace (``chrome://tracing``/Perfetto) events for one process row."""
    thread_ids: dict[str, int] = {}
    body = []
    for s in spans:
        tid = thread_ids.setdefault(s.thread, len(thread_ids))
        label = s.category if s.microbatch is None else f"{s.category} mb{s.microbatch}"
        meta = {"step": s.step, "microbatch": s.microbatch}
        meta.update(s.args or {})
        body.append({"name": label, "cat": s.category, "ph": "X", "pid": pid, "tid": tid,
                     "ts": s.start * 1e6, "dur": s.duration * 1e6, "args": meta})
    head = [{"ph": "M", "name": "process_name", "pid": pid, "args": {"name": process_label}}]
    head += [{"ph": "M", "name": "thread_name", "pid": pid, "tid": tid, "args": {"name": name}}
             for name, tid in thread_ids.items()]
    return head + body


class Timeline:
    """Thread-safe span log of one stage process."""

    def __init__(self, worker: str = "local", stage: int = 0, enabled: bool = True):
        self.worker = worker
        self.stage = stage
        self.enabled = enabled
        # wall-clock origin + a monotonic offset: spans from several processes line up on
        # one trace, and a clock step during the run does not reorder this process's spans
        self._origin = time.time() - time.perf_counter()
        self._log: list[Span] = []
        self._mu = threading.Lock()

    def now(self) -> float:
        return self._origin + time.perf_counter()

    def _append(self, span: Span) -> None:
        with self._mu:
            self._log.append(span)

    def add(self, category: str, start: float, end: float, step=None, microbatch=None, **args) -> None:
        if self.enabled:
            self._append(Span(category, start, end, threading.current_thread().name, step, microbatch,
                              args or None))

    def span(self, category: str, step=None, microbatch=None, **args):
        """Context manager recording the time spent inside it under ``category``."""
        return _Measured(self, category, step, microbatch, args)

    def add_device_spans(self, spans: list[dict], step: int, step_start_wall: float, thread: str = "gpu") -> None:
        """Record CUDA-event spans given as millisecond offsets from the step start."""
        for s in spans:
            self._append(Span(s["cat"], step_start_wall + s["start_ms"] * 1e-3, step_start_wall + s["end_ms"] * 1e-3,
                              thread, step, s.get("mb"), {"device": True}))

    def spans(self, step: int | None = None) -> list[Span]:
        with self._mu:
            snapshot = list(self._log)
        return snapshot if step is None else [s for s in snapshot if s.step == step]

    def drop_before(self, t: float) -> None:
        """Forget spans that ended before ``t`` (keeps the log bounded over long runs)."""
        with self._mu:
            self._log = [s for s in self._log if s.end >= t]

    def step_metrics(self, step: int, window: tuple[float, float]) -> dict:
        lo, hi = window
        clipped = [s._replace(start=max(s.start, lo), end=min(s.end, hi)) for s in self.spans()
                   if s.end > lo and s.start < hi]
        tally = sweep([(s.start, s.end, _GROUP[s.category]) for s in clipped if s.category in _GROUP])
        compute_s = sum(v for k, v in tally.items() if "compute" in k)
        comm_s = sum(v for k, v in tally.items() if "comm" in k)
        both_s = tally.get(frozenset(("compute", "comm")), 0.0)
        phases: dict[str, float] = defaultdict(float)
        for s in clipped:
            # work spans of a neighbouring step that fall inside the window still occupy it;
            # waits and queueing are attributed to their own step only
            if s.step == step or s.category in _GROUP:
                phases[s.category] += s.duration
        return {"compute_s": compute_s, "communication_s": comm_s, "overlapped_s": both_s,
                "exposed_communication_s": comm_s - both_s,
                "idle_s": max(0.0, (hi - lo) - sum(tally.values())),
                "overlap_ratio": both_s / comm_s if comm_s > 0 else 0.0, "phase_s": dict(phases)}

    def to_chrome_events(self, pid: int | None = None) -> list[dict]:
        return chrome_events(self.spans(), self.stage if pid is None else pid, f"stage {self.stage} · {self.worker}")

    def export(self) -> list[dict]:
        return [s.as_dict() for s in self.spans()]


class _Measured:
    __slots__ = ("tl", "category", "step", "microbatch", "args", "t0")

    def __init__(self, tl: Timeline, category: str, step, microbatch, args: dict):
        self.tl, self.category, self.step, self.microbatch, self.args = tl, category, step, microbatch, args

    def __enter__(self):
        self.t0 = self.tl.now()
        return self

    def __exit__(self, *exc):
        self.tl.add(self.category, self.t0, self.tl.now(), self.step, self.microbatch, **self.args)
        return False


def write_chrome_trace(path, stage_events: list[list[dict]]) -> Path:
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    merged = [ev for events in stage_events for ev in events]
    out.write_text(json.dumps({"traceEvents": merged, "displayTimeUnit": "ms"}))
    return out


def chrome_events_from_export(spans: list[dict], stage: int, worker: str) -> list[dict]:
    """Chrome events for spans exported by another process (``Timeline.export``)."""
    rows = [Span(d["category"], d["start"], d["end"], d.get("thread", "main"), d.get("step"), d.get("microbatch"),
                 d.get("args")) for d in spans]
    return chrome_events(rows, stage, f"stage {stage} · {worker}")

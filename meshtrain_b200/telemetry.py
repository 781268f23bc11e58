"""Event log lines, JSONL mirrors and metrics files (reference telemetry.py:23-100).

    [HH:MM:SS.mmm] worker=<w> job=<j> step=<s> mb=<m> EVENT k=v ...

``MESHTRAIN_QUIET=1`` silences stdout; ``MetricsWriter`` appends one JSON
record per line to ``metrics.jsonl``.
"""

from __future__ import annotations

import json
import os
import sys
import threading
import time
import uuid
from datetime import datetime
from pathlib import Path


def new_run_id(prefix: str = "run") -> str:
    return f"{prefix}-{datetime.now().strftime('%Y%m%d-%H%M%S')}-{uuid.uuid4().hex[:6]}"


def _fmt(k: str, v) -> str:
    if isinstance(v, float):
        if k.endswith("_s"):
            return f"{k[:-2]}_ms={v * 1e3:.2f}"
        return f"{k}={v:.6g}"
    if isinstance(v, int) and (k.endswith("bytes") or k == "output"):
        return f"{k}={v / 1e6:.2f}MB" if v >= 1e6 else f"{k}={v}B"
    return f"{k}={v}"


class EventLogger:
    def __init__(self, worker: str = "local", job: str | None = None, jsonl_path: str | Path | None = None,
                 stream=None):
        self.worker, self.job = worker, job
        self.quiet = os.environ.get("MESHTRAIN_QUIET", "") not in ("", "0")
        self.stream = stream or sys.stdout
        self._lock = threading.Lock()
        self._jsonl = None
        if jsonl_path:
            p = Path(jsonl_path)
            p.parent.mkdir(parents=True, exist_ok=True)
            self._jsonl = open(p, "a")

    def format(self, event: str, step, mb, **fields) -> str:
        ts = datetime.now().strftime("%H:%M:%S.%f")[:-3]
        parts = [f"[{ts}]", f"worker={self.worker}"]
        if self.job:
            parts.append(f"job={self.job}")
        if step is not None:
            parts.append(f"step={step}")
        if mb is not None:
            parts.append(f"mb={mb}")
        parts.append(event)
        parts += [_fmt(k, v) for k, v in fields.items()]
        return " ".join(parts)

    def log(self, event: str, step=None, mb=None, **fields) -> str:
        line = self.format(event, step, mb, **fields)
        with self._lock:
            if not self.quiet:
                print(line, file=self.stream, flush=True)
            if self._jsonl is not None:
                rec = {"ts": time.time(), "worker": self.worker, "job": self.job, "step": step, "mb": mb,
                       "event": event, **fields}
                self._jsonl.write(json.dumps(rec, default=str) + "\n")
                self._jsonl.flush()
        return line

    def close(self) -> None:
        if self._jsonl is not None:
            self._jsonl.close()
            self._jsonl = None


class MetricsWriter:
    def __init__(self, path: str | Path):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self._lock = threading.Lock()

    def write(self, record: dict) -> None:
        with self._lock, open(self.path, "a") as f:
            f.write(json.dumps(record, default=str) + "\n")

    def read(self) -> list[dict]:
        if not self.path.exists():
            return []
        return [json.loads(line) for line in self.path.read_text().splitlines() if line.strip()]


def read_jsonl(path) -> list[dict]:
    """Records of a JSON-lines file; a torn last line (writer still running) is skipped."""
    p = Path(path)
    if not p.exists():
        return []
    out = []
    for line in p.read_text().splitlines():
        if line.strip():
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                continue
    return out

"""What the coordinator remembers about workers and jobs (in memory only).

A restarted coordinator starts empty: workers notice (their heartbeat gets a
404) and register again, and finished jobs remain readable in their run
directories.  ``public()`` gives the JSON a record shows on the HTTP API; its
keys are the API's (reference coordinator/state.py:11-96).
"""

from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field
from typing import Any


class WorkerStatus(str, enum.Enum):
    ONLINE = "ONLINE"
    BUSY = "BUSY"
    OFFLINE = "OFFLINE"


class JobStatus(str, enum.Enum):
    PLANNED = "PLANNED"
    RUNNING = "RUNNING"
    COMPLETED = "COMPLETED"
    FAILED = "FAILED"
    STOPPED = "STOPPED"


def _now() -> float:
    return time.time()


@dataclass
class WorkerRecord:
    worker_id: str
    name: str
    hardware: dict
    backend: str
    device_info: dict
    data_host: str
    data_port: int
    status: WorkerStatus = WorkerStatus.ONLINE
    registered_at: float = field(default_factory=_now)
    last_heartbeat: float = field(default_factory=_now)
    memory: dict = field(default_factory=dict)
    benchmark: dict | None = None
    current_job: str | None = None
    capabilities: dict = field(default_factory=dict)

    # API key -> hardware dict key
    HARDWARE_FIELDS = {"hostname": "hostname", "platform": "platform", "cpu_count": "cpu_count",
                       "ram_total": "ram_total"}

    @property
    def host_key(self) -> str:
        """Workers with equal keys share a box, so their GPUs can use NCCL over NVLink."""
        hw = self.hardware
        return str(hw.get("host_id") or hw.get("hostname") or self.data_host)

    def public(self) -> dict:
        out = {key: self.hardware.get(src) for key, src in self.HARDWARE_FIELDS.items()}
        out.update(
            worker_id=self.worker_id, name=self.name, accelerators=self.hardware.get("accelerators", []),
            capabilities=self.hardware.get("capabilities", []), backend=self.backend, device=self.device_info,
            data_address=f"{self.data_host}:{self.data_port}", status=self.status.value,
            last_heartbeat_age_s=round(_now() - self.last_heartbeat, 1), memory=self.memory,
            benchmark=self.benchmark, current_job=self.current_job, device_capabilities=self.capabilities,
            host=self.host_key)
        return out


@dataclass
class JobRecord:
    job_id: str
    config: dict
    plan: dict
    status: JobStatus = JobStatus.PLANNED
    error: str | None = None
    created_at: float = field(default_factory=_now)
    finished_at: float | None = None
    stage_workers: list[str] = field(default_factory=list)
    stages_done: dict[int, dict] = field(default_factory=dict)
    losses: list[tuple[int, float]] = field(default_factory=list)
    last_metrics: dict[int, dict] = field(default_factory=dict)
    run_dir: str = ""
    summary: dict | None = None
    attempt: int = 0
    attempts: list[dict] = field(default_factory=list)
    budget_overrides: dict[str, int] = field(default_factory=dict)
    memory_reports: dict[str, dict] = field(default_factory=dict)
    timelines: dict[int, tuple[str, list]] = field(default_factory=dict)  # large: kept off the API

    PUBLIC = ("job_id", "error", "plan", "stage_workers", "losses", "last_metrics", "stages_done", "run_dir",
              "summary", "attempt", "attempts", "memory_reports", "created_at", "finished_at")

    @property
    def name(self) -> str | None:
        return self.config.get("job", {}).get("name")

    def public(self) -> dict[str, Any]:
        out = {key: getattr(self, key) for key in self.PUBLIC}
        out.update(name=self.name, status=self.status.value)
        return out

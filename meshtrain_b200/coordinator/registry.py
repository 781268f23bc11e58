"""Worker registry: ids, liveness from heartbeats, per-worker command mailboxes.

Covers the reference's registry (coordinator/registry.py:18-110): stable worker
ids, liveness from heartbeats with offline callbacks, and a long-poll command
queue per worker.  Here every worker has its own ``_Mailbox`` with its own
condition variable, so a command wakes only the worker it is for; ``poll``
blocks up to ``timeout`` for the first command and then drains everything
queued, so one long-poll round trip carries a burst.
"""

from __future__ import annotations

import collections
import re
import threading
import time
import uuid
from typing import Callable

from meshtrain_b200.coordinator.state import WorkerRecord, WorkerStatus


def slug(name: str) -> str:
    """A worker name reduced to characters safe in ids, file names and URLs."""
    cleaned = re.sub(r"[^A-Za-z0-9_.-]+", "-", name).strip("-")
    return cleaned[:48] or "worker"


class _Mailbox:
    def __init__(self):
        self._queue: collections.deque[dict] = collections.deque()
        self._ready = threading.Condition()

    def put(self, command: dict) -> None:
        with self._ready:
            self._queue.append(command)
            self._ready.notify()

    def take_all(self, timeout: float) -> list[dict]:
        with self._ready:
            if not self._queue:
                self._ready.wait_for(lambda: bool(self._queue), timeout=max(0.0, timeout))
            taken = list(self._queue)
            self._queue.clear()
        return taken


class WorkerRegistry:
    def __init__(self, heartbeat_timeout_s: float = 15.0):
        self.heartbeat_timeout_s = heartbeat_timeout_s
        self.on_offline: list[Callable[[WorkerRecord], None]] = []
        self._records: dict[str, WorkerRecord] = {}
        self._boxes: dict[str, _Mailbox] = {}
        self._mu = threading.Lock()

    def _returning(self, name: str, data_host: str, data_port: int) -> WorkerRecord | None:
        """The record of a worker that registered before from the same name and data endpoint."""
        return next((r for r in self._records.values()
                     if r.name == name and r.data_host == data_host and r.data_port == data_port), None)

    def _fresh_id(self, base: str) -> str:
        wid = base
        while wid in self._records:
            wid = f"{base}-{uuid.uuid4().hex[:4]}"
        return wid

    def register(self, *, name: str, hardware: dict, backend: str, device_info: dict, data_host: str,
                 data_port: int, capabilities: dict | None = None) -> WorkerRecord:
        """Adds a worker, or revives the record of a restarted one (same name and data endpoint)."""
        base = slug(name)
        caps = dict(capabilities or {})
        with self._mu:
            rec = self._returning(base, data_host, data_port)
            if rec is None:
                wid = self._fresh_id(base)
                rec = WorkerRecord(wid, wid, hardware, backend, device_info, data_host, data_port, capabilities=caps)
                self._records[wid] = rec
                self._boxes[wid] = _Mailbox()
                return rec
            rec.hardware, rec.backend, rec.device_info, rec.capabilities = hardware, backend, device_info, caps
            rec.status, rec.current_job, rec.last_heartbeat = WorkerStatus.ONLINE, None, time.time()
            return rec

    def get(self, worker_id: str) -> WorkerRecord | None:
        with self._mu:
            return self._records.get(worker_id)

    def all(self) -> list[WorkerRecord]:
        with self._mu:
            return list(self._records.values())

    def online(self) -> list[WorkerRecord]:
        """Workers not marked offline (busy ones included)."""
        return [r for r in self.all() if r.status is not WorkerStatus.OFFLINE]

    def idle(self) -> list[WorkerRecord]:
        return [r for r in self.all() if r.status is WorkerStatus.ONLINE]

    def heartbeat(self, worker_id: str, memory: dict | None = None) -> bool:
        """Records a sign of life; False for an unknown id (the worker must register again)."""
        with self._mu:
            rec = self._records.get(worker_id)
            if rec is None:
                return False
            rec.last_heartbeat = time.time()
            rec.memory = memory or rec.memory
            if rec.status is WorkerStatus.OFFLINE:
                rec.status = WorkerStatus.ONLINE
        return True

    def check_liveness(self, now: float | None = None) -> list[WorkerRecord]:
        """Marks workers silent for longer than the timeout offline and runs the callbacks for them."""
        cutoff = (time.time() if now is None else now) - self.heartbeat_timeout_s
        with self._mu:
            lost = [r for r in self._records.values()
                    if r.status is not WorkerStatus.OFFLINE and r.last_heartbeat < cutoff]
            for rec in lost:
                rec.status = WorkerStatus.OFFLINE
        for rec in lost:  # outside the lock: callbacks call back into the registry
            for callback in self.on_offline:
                callback(rec)
        return lost

    def _box(self, worker_id: str) -> _Mailbox:
        with self._mu:
            box = self._boxes.get(worker_id)
        if box is None:
            raise KeyError(worker_id)
        return box

    def send(self, worker_id: str, command: dict) -> None:
        self._box(worker_id).put(command)

    def poll(self, worker_id: str, timeout: float) -> list[dict]:
        """Commands queued for the worker, waiting up to ``timeout`` seconds for the first one."""
        return self._box(worker_id).take_all(timeout)

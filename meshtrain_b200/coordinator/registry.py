"""Worker registry: ids, liveness from heartbeats, per-worker command mailboxes.

(reference coordinator/registry.py:18-110.)  A mailbox is a list guarded by a
condition variable; ``poll`` blocks up to ``timeout`` for the first command and
then drains everything queued, so one long-poll round trip can carry a burst.
"""

from __future__ import annotations

import re
import threading
import time
import uuid
from typing import Callable

from meshtrain_b200.coordinator.state import WorkerRecord, WorkerStatus


def slug(name: str) -> str:
    s = re.sub(r"[^A-Za-z0-9_.-]+", "-", name).strip("-")
    return s[:48] or "worker"


class WorkerRegistry:
    def __init__(self, heartbeat_timeout_s: float = 15.0):
        self.heartbeat_timeout_s = heartbeat_timeout_s
        self._workers: dict[str, WorkerRecord] = {}
        self._mail: dict[str, list[dict]] = {}
        self._cv = threading.Condition(threading.RLock())
        self.on_offline: list[Callable[[WorkerRecord], None]] = []

    def register(self, *, name: str, hardware: dict, backend: str, device_info: dict, data_host: str,
                 data_port: int, capabilities: dict | None = None) -> WorkerRecord:
        base = slug(name)
        with self._cv:
            for w in self._workers.values():  # a restarted worker keeps its id
                if w.name == base and (w.data_host, w.data_port) == (data_host, data_port):
                    w.hardware, w.backend, w.device_info = hardware, backend, device_info
                    w.capabilities = capabilities or {}
                    w.status, w.last_heartbeat, w.current_job = WorkerStatus.ONLINE, time.time(), None
                    return w
            wid = base
            while wid in self._workers:
                wid = f"{base}-{uuid.uuid4().hex[:4]}"
            rec = WorkerRecord(wid, wid, hardware, backend, device_info, data_host, data_port,
                               capabilities=capabilities or {})
            self._workers[wid] = rec
            self._mail[wid] = []
            return rec

    def get(self, worker_id: str) -> WorkerRecord | None:
        with self._cv:
            return self._workers.get(worker_id)

    def all(self) -> list[WorkerRecord]:
        with self._cv:
            return list(self._workers.values())

    def online(self) -> list[WorkerRecord]:
        return [w for w in self.all() if w.status is not WorkerStatus.OFFLINE]

    def idle(self) -> list[WorkerRecord]:
        return [w for w in self.all() if w.status is WorkerStatus.ONLINE]

    def heartbeat(self, worker_id: str, memory: dict | None = None) -> bool:
        with self._cv:
            w = self._workers.get(worker_id)
            if w is None:
                return False
            w.last_heartbeat = time.time()
            if memory:
                w.memory = memory
            if w.status is WorkerStatus.OFFLINE:
                w.status = WorkerStatus.ONLINE
            return True

    def check_liveness(self, now: float | None = None) -> list[WorkerRecord]:
        now = time.time() if now is None else now
        with self._cv:
            gone = [w for w in self._workers.values()
                    if w.status is not WorkerStatus.OFFLINE and now - w.last_heartbeat > self.heartbeat_timeout_s]
            for w in gone:
                w.status = WorkerStatus.OFFLINE
        for w in gone:
            for cb in self.on_offline:
                cb(w)
        return gone

    def send(self, worker_id: str, command: dict) -> None:
        with self._cv:
            if worker_id not in self._mail:
                raise KeyError(worker_id)
            self._mail[worker_id].append(command)
            self._cv.notify_all()

    def poll(self, worker_id: str, timeout: float) -> list[dict]:
        deadline = time.monotonic() + max(0.0, timeout)
        with self._cv:
            if worker_id not in self._mail:
                raise KeyError(worker_id)
            box = self._mail[worker_id]
            while not box:
                left = deadline - time.monotonic()
                if left <= 0:
                    return []
                self._cv.wait(left)
            out = list(box)
            box.clear()
            return out

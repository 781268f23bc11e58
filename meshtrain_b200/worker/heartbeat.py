"""Worker liveness: a timer thread that reports to the coordinator every ``interval_s``.

Each beat carries the worker's memory snapshot.  A 404 means the coordinator
has restarted and no longer knows the worker, so ``on_unknown`` registers it
again; any other failure is counted and handed to ``on_error``, never raised
(the coordinator marks a worker OFFLINE only after its heartbeat timeout).
Same behaviour as the reference (worker/heartbeat.py:10-50).
"""

from __future__ import annotations

import threading
from typing import Callable

import httpx


class Heartbeat:
    def __init__(self, client, worker_id_fn: Callable[[], str | None], memory_fn: Callable[[], dict],
                 interval_s: float = 3.0, on_unknown: Callable[[], None] | None = None,
                 on_error: Callable[[Exception], None] | None = None):
        self.client = client
        self.worker_id_fn = worker_id_fn
        self.memory_fn = memory_fn
        self.interval_s = interval_s
        self.on_unknown = on_unknown
        self.on_error = on_error
        self.beats = 0
        self.failures = 0
        self._halt = threading.Event()
        self._timer = threading.Thread(target=self._run, daemon=True, name="heartbeat")

    def start(self) -> "Heartbeat":
        self._timer.start()
        return self

    def _failed(self, exc: Exception) -> None:
        self.failures += 1
        forgotten = isinstance(exc, httpx.HTTPStatusError) and exc.response.status_code == 404
        callback = self.on_unknown if forgotten else self.on_error
        if callback is None:
            return
        callback() if forgotten else callback(exc)

    def beat(self) -> None:
        """Sends one heartbeat now (no-op until the worker has an id)."""
        worker_id = self.worker_id_fn()
        if worker_id is None:
            return
        try:
            self.client.heartbeat(worker_id, {"memory": self.memory_fn()})
        except httpx.HTTPError as exc:
            self._failed(exc)
            return
        self.beats += 1
        self.failures = 0

    def _run(self) -> None:
        while not self._halt.wait(self.interval_s):
            self.beat()

    def stop(self) -> None:
        self._halt.set()

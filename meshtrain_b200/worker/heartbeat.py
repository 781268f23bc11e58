"""Background heartbeat: liveness + memory snapshot every ``interval_s`` (reference worker/heartbeat.py:10-50).

A 404 means the coordinator restarted and forgot this worker: ``on_unknown``
re-registers.  Other failures are counted and reported, never raised.
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
        self.failures = 0
        self.beats = 0
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, daemon=True, name="heartbeat")

    def start(self) -> "Heartbeat":
        self._thread.start()
        return self

    def beat(self) -> None:
        wid = self.worker_id_fn()
        if wid is None:
            return
        try:
            self.client.heartbeat(wid, {"memory": self.memory_fn()})
            self.failures = 0
            self.beats += 1
        except httpx.HTTPStatusError as exc:
            self.failures += 1
            if exc.response.status_code == 404 and self.on_unknown is not None:
                self.on_unknown()
            elif self.on_error is not None:
                self.on_error(exc)
        except httpx.HTTPError as exc:
            self.failures += 1
            if self.on_error is not None:
                self.on_error(exc)

    def _loop(self) -> None:
        while not self._stop.wait(self.interval_s):
            self.beat()

    def stop(self) -> None:
        self._stop.set()

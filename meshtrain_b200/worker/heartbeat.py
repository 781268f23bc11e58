"""Worker liveness: a daemon thread that reports to the coordinator at a fixed period.

What one report contains is the caller's business (``send``: the agent sends its
worker id and a memory snapshot).  A 404 answer means the coordinator restarted
and no longer knows the worker, so ``forgotten`` runs (the agent registers
again); any other HTTP failure is counted and passed to ``failed``, never
raised: the coordinator marks a worker offline only after its own heartbeat
timeout.  Behaviour of the reference's heartbeat (worker/heartbeat.py:10-50).
"""

from __future__ import annotations

import threading
from typing import Callable

import httpx


class Heartbeat:
    def __init__(self, send: Callable[[], bool], *, every_s: float = 3.0,
                 forgotten: Callable[[], None] | None = None, failed: Callable[[Exception], None] | None = None):
        """``send`` makes one report and returns False when there is nothing to report yet."""
        self._send = send
        self.every_s = every_s
        self._forgotten = forgotten
        self._failed = failed
        self.sent = 0
        self.consecutive_failures = 0
        self._halt = threading.Event()
        self._thread = threading.Thread(target=self._loop, daemon=True, name="heartbeat")

    def start(self) -> "Heartbeat":
        self._thread.start()
        return self

    def beat(self) -> None:
        """One report now (also what the background thread does every period)."""
        try:
            delivered = self._send()
        except httpx.HTTPStatusError as exc:
            self.consecutive_failures += 1
            if exc.response.status_code == 404:
                if self._forgotten is not None:
                    self._forgotten()
            elif self._failed is not None:
                self._failed(exc)
            return
        except httpx.HTTPError as exc:
            self.consecutive_failures += 1
            if self._failed is not None:
                self._failed(exc)
            return
        if delivered:
            self.sent += 1
            self.consecutive_failures = 0

    def _loop(self) -> None:
        while not self._halt.wait(self.every_s):
            self.beat()

    def stop(self) -> None:
        self._halt.set()

"""Reusable host staging buffers keyed by (shape, dtype, pinned).

Steady-state microbatches stop allocating: ``acquire`` reuses an idle buffer,
``release(buf, event)`` returns it (deferred until ``event`` has completed,
e.g. an async H2D copy).  Pinned memory falls back to pageable if pinning
fails; idle memory is capped per key and in total so dynamic shapes cannot grow
the pool without bound (reference runtime/buffers.py:30-108).
"""

from __future__ import annotations

import threading
from collections import defaultdict

import torch


class BufferPool:
    def __init__(self, *, pinned: bool = False, enabled: bool = True, max_free_per_key: int = 8,
                 max_bytes: int = 2 * 1024 ** 3):
        self.pinned = pinned
        self.enabled = enabled
        self.max_free_per_key = max_free_per_key
        self.max_bytes = max_bytes
        self._idle: dict[tuple, list[torch.Tensor]] = defaultdict(list)
        self._pending: list[tuple[torch.Tensor, object]] = []
        self._lock = threading.Lock()
        self.allocation_count = 0
        self.reuse_count = 0
        self.pinned_fallbacks = 0
        self.bytes_reserved = 0
        self.bytes_allocated = 0

    @staticmethod
    def _key(t: torch.Tensor) -> tuple:
        return (tuple(t.shape), t.dtype, t.is_pinned())

    def _new(self, shape, dtype) -> torch.Tensor:
        t = None
        if self.pinned:
            try:
                t = torch.empty(shape, dtype=dtype, pin_memory=True)
            except RuntimeError:
                self.pinned_fallbacks += 1
        if t is None:
            t = torch.empty(shape, dtype=dtype)
        self.allocation_count += 1
        self.bytes_allocated += t.numel() * t.element_size()
        return t

    def _retire_pending(self) -> None:
        keep = []
        for buf, ev in self._pending:
            if ev is None or ev.query():
                self._stash(buf)
            else:
                keep.append((buf, ev))
        self._pending = keep

    def _stash(self, buf: torch.Tensor) -> None:
        key = self._key(buf)
        n = buf.numel() * buf.element_size()
        if len(self._idle[key]) < self.max_free_per_key and self.bytes_reserved + n <= self.max_bytes:
            self._idle[key].append(buf)
            self.bytes_reserved += n

    def acquire(self, shape, dtype: torch.dtype) -> torch.Tensor:
        shape = tuple(shape)
        if not self.enabled:
            return self._new(shape, dtype)
        with self._lock:
            self._retire_pending()
            for pinned in ((True, False) if self.pinned else (False,)):
                idle = self._idle.get((shape, dtype, pinned))
                if idle:
                    buf = idle.pop()
                    self.bytes_reserved -= buf.numel() * buf.element_size()
                    self.reuse_count += 1
                    return buf
            return self._new(shape, dtype)

    def release(self, buf: torch.Tensor | None, event=None) -> None:
        if not self.enabled or buf is None:
            return
        with self._lock:
            if event is None:
                self._stash(buf)
            else:
                self._pending.append((buf, event))

    def stats(self) -> dict:
        with self._lock:
            return {"allocation_count": self.allocation_count, "reuse_count": self.reuse_count,
                    "bytes_reserved": self.bytes_reserved, "bytes_allocated": self.bytes_allocated,
                    "pinned": self.pinned, "pinned_fallbacks": self.pinned_fallbacks, "deferred": len(self._pending)}

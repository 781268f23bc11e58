"""Host staging memory for the host pipeline, recycled as byte slabs.

Every buffer the pool hands out is a typed view of a ``uint8`` slab whose size
is rounded up to a size class (powers of two split into eight steps, so at
most 12.5 % is wasted).  A slab returns to the idle list of its class when the
caller releases the view, and any later request of that class reuses it,
whatever its shape or dtype: the last, shorter microbatch of a step and a
tensor of another dtype of similar size share memory instead of each keeping
their own.  This is the reference's staging pool (runtime/buffers.py:30-108)
organised by size instead of by ``(shape, dtype)``.

* ``pinned=True`` asks for page-locked slabs (for asynchronous CUDA copies);
  when pinning fails the pool falls back to pageable memory and counts it in
  ``pinned_fallbacks``.
* ``release(buf, event)`` keeps the slab out of circulation until ``event``
  reports completion (``event.query()``), e.g. an asynchronous host-to-device
  copy that still reads it.  Fenced slabs are retired in release order.
* At most ``max_idle_per_class`` idle slabs per class and ``max_bytes`` idle
  bytes in total are kept; a release beyond either cap drops the slab.
"""

from __future__ import annotations

import threading
from collections import deque

import torch

MIN_SLAB = 256


def size_class(nbytes: int) -> int:
    """Smallest class >= nbytes: multiples of 1/8 of the enclosing power of two."""
    if nbytes <= MIN_SLAB:
        return MIN_SLAB
    top = 1 << (nbytes - 1).bit_length()  # next power of two
    step = max(MIN_SLAB, top // 16)       # classes between top/2 and top in steps of top/16
    return -(-nbytes // step) * step


class BufferPool:
    def __init__(self, *, pinned: bool = False, enabled: bool = True, max_idle_per_class: int = 8,
                 max_bytes: int = 2 * 1024 ** 3):
        self.pinned = pinned
        self.enabled = enabled
        self.max_idle_per_class = max_idle_per_class
        self.max_bytes = max_bytes
        self._idle: dict[int, list[torch.Tensor]] = {}
        self._owner: dict[int, torch.Tensor] = {}      # data_ptr of a handed-out view -> its slab
        self._fenced: deque[tuple[torch.Tensor, object]] = deque()
        self._lock = threading.Lock()
        self.allocation_count = 0
        self.reuse_count = 0
        self.pinned_fallbacks = 0
        self.bytes_reserved = 0    # bytes held in idle slabs
        self.bytes_allocated = 0   # bytes of every slab ever allocated

    def _new_slab(self, nbytes: int) -> torch.Tensor:
        slab = None
        if self.pinned:
            try:
                slab = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            except RuntimeError:
                self.pinned_fallbacks += 1
        if slab is None:
            slab = torch.empty(nbytes, dtype=torch.uint8)
        self.allocation_count += 1
        self.bytes_allocated += nbytes
        return slab

    def _retire_fenced(self) -> None:
        while self._fenced and (self._fenced[0][1] is None or self._fenced[0][1].query()):
            self._keep_idle(self._fenced.popleft()[0])

    def _keep_idle(self, slab: torch.Tensor) -> None:
        n = slab.numel()
        idle = self._idle.setdefault(n, [])
        if len(idle) < self.max_idle_per_class and self.bytes_reserved + n <= self.max_bytes:
            idle.append(slab)
            self.bytes_reserved += n

    def acquire(self, shape, dtype: torch.dtype) -> torch.Tensor:
        shape = tuple(int(d) for d in shape)
        numel = 1
        for d in shape:
            numel *= d
        nbytes = numel * dtype.itemsize
        if not self.enabled:
            return torch.empty(shape, dtype=dtype)
        cls = size_class(nbytes)
        with self._lock:
            self._retire_fenced()
            idle = self._idle.get(cls)
            if idle:
                slab = idle.pop()
                self.bytes_reserved -= cls
                self.reuse_count += 1
            else:
                slab = self._new_slab(cls)
            view = slab[:nbytes].view(dtype).view(shape)
            self._owner[view.data_ptr()] = slab
            return view

    def release(self, buf: torch.Tensor | None, event=None) -> None:
        if not self.enabled or buf is None:
            return
        with self._lock:
            slab = self._owner.pop(buf.data_ptr(), None)
            if slab is None:
                return  # not one of ours (or released twice)
            if event is None:
                self._keep_idle(slab)
            else:
                self._fenced.append((slab, event))

    def stats(self) -> dict:
        with self._lock:
            return {"allocation_count": self.allocation_count, "reuse_count": self.reuse_count,
                    "bytes_reserved": self.bytes_reserved, "bytes_allocated": self.bytes_allocated,
                    "pinned": self.pinned, "pinned_fallbacks": self.pinned_fallbacks, "deferred": len(self._fenced)}

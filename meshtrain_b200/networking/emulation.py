"""Link emulation for experiments: each direction behaves like latency + bytes/bandwidth.

Wraps any Transport; a lock per direction serialises frames like a real wire
(reference networking/emulation.py:29-79).  Used only in experiments/tests and
always labelled as emulated in their output.
"""

from __future__ import annotations

import threading
import time

from meshtrain_b200.networking.transport import Transport


class EmulatedLink(Transport):
    def __init__(self, inner: Transport, bandwidth_bytes_per_s: float, latency_s: float = 0.0):
        super().__init__(inner.max_payload_bytes)
        if bandwidth_bytes_per_s <= 0:
            raise ValueError("bandwidth must be positive")
        self.inner = inner
        self.bandwidth = float(bandwidth_bytes_per_s)
        self.latency = float(latency_s)
        self._tx = threading.Lock()

    @property
    def payload_allocator(self):
        return getattr(self.inner, "payload_allocator", None)

    @payload_allocator.setter
    def payload_allocator(self, fn):
        if hasattr(self, "inner"):
            self.inner.payload_allocator = fn

    def wire_time(self, nbytes: int) -> float:
        return self.latency + nbytes / self.bandwidth

    def _send_frame(self, frame) -> None:  # pragma: no cover - send_packet is overridden
        self.inner._send_frame(frame)

    def send_packet(self, packet) -> float:
        t0 = time.perf_counter()
        with self._tx:
            nbytes = len(packet.payload) + 256
            target = t0 + self.wire_time(nbytes)
            self.inner.send_packet(packet)
            delay = target - time.perf_counter()
            if delay > 0:
                time.sleep(delay)
        self.bytes_sent += len(packet.payload)
        return time.perf_counter() - t0

    def _recv_packet(self, timeout):
        pkt = self.inner.recv_packet(timeout)
        self.last_frame_s = getattr(self.inner, "last_frame_s", 0.0)
        return pkt, len(pkt.payload)

    def close(self) -> None:
        self.inner.close()

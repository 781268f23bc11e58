"""Link emulation for experiments: each direction behaves like latency + bytes/bandwidth.

``EmulatedLink`` wraps any link and holds every send until the frame would
have crossed a wire of the given bandwidth and latency; one lock per direction
serialises frames the way a real wire does.  Same model as the reference's
emulated link (networking/emulation.py:29-79).  Used only by experiments and
tests, whose output says the link was emulated.
"""

from __future__ import annotations

import threading
import time

from meshtrain_b200.networking.transport import PacketLink

# Bytes of framing (prefix + JSON header) charged per packet on the emulated wire.
FRAME_OVERHEAD_BYTES = 256


class EmulatedLink(PacketLink):
    def __init__(self, inner, bandwidth_bytes_per_s: float, latency_s: float = 0.0):
        if bandwidth_bytes_per_s <= 0:
            raise ValueError("bandwidth must be positive")
        self.inner = inner
        self.bandwidth = float(bandwidth_bytes_per_s)
        self.latency = float(latency_s)
        self.bytes_sent = 0
        self._wire = threading.Lock()

    # the receive side, the allocator hook and the limits are the inner link's
    @property
    def payload_allocator(self):
        return self.inner.payload_allocator

    @payload_allocator.setter
    def payload_allocator(self, fn):
        self.inner.payload_allocator = fn

    @property
    def max_payload_bytes(self) -> int:
        return self.inner.max_payload_bytes

    @property
    def bytes_received(self) -> int:
        return self.inner.bytes_received

    @property
    def last_frame_s(self) -> float:
        return self.inner.last_frame_s

    @property
    def peer(self) -> str:
        return f"emulated({getattr(self.inner, 'peer', '?')})"

    def wire_time(self, nbytes: int) -> float:
        return self.latency + nbytes / self.bandwidth

    def send_packet(self, packet) -> float:
        t0 = time.perf_counter()
        with self._wire:
            done_at = t0 + self.wire_time(len(packet.payload) + FRAME_OVERHEAD_BYTES)
            self.inner.send_packet(packet)
            remaining = done_at - time.perf_counter()
            if remaining > 0:
                time.sleep(remaining)
        self.bytes_sent += len(packet.payload)
        return time.perf_counter() - t0

    def recv_packet(self, timeout: float | None = None):
        return self.inner.recv_packet(timeout)

    def close(self) -> None:
        self.inner.close()

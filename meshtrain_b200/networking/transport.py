"""Point-to-point packet transports between pipeline peers.

A ``Transport`` is an ordered, reliable, bidirectional packet channel with
byte accounting; it never sees torch devices.  ``PipeTransport`` wraps a
multiprocessing connection (stages as processes on one host); ``TCPTransport``
(networking/tcp.py) is the network data plane.  GPU stages inside one box use
NCCL instead (parallel/p2p.py).  Behaviour follows reference
networking/transport.py:52-170, including the optional in-place receive hook.
"""

from __future__ import annotations

import abc
import math
import threading
import time

import torch

from meshtrain_b200.networking.packet import WIRE_DTYPES, MessageType, TensorPacket
from meshtrain_b200.networking.protocol import (
    DEFAULT_MAX_PAYLOAD_BYTES, PREFIX_SIZE, ProtocolError, decode_packet, encode_head)
from meshtrain_b200.networking.serialization import TensorLifecycle, packet_to_tensor, tensor_to_packet


class TransportError(RuntimeError):
    pass


class TransportTimeout(TransportError, TimeoutError):
    pass


class TransportClosed(TransportError, ConnectionError):
    pass


class Transport(abc.ABC):
    def __init__(self, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES):
        self.max_payload_bytes = max_payload_bytes
        self.bytes_sent = 0
        self.bytes_received = 0
        self.last_frame_s = 0.0
        self._send_lock = threading.Lock()
        # Optional fn(message_type, torch_dtype, shape) -> CPU tensor to receive into.
        self.payload_allocator = None

    def _allocate(self, header, payload_len: int):
        """A receive buffer matching an (untrusted) header exactly, or None."""
        fn = self.payload_allocator
        if fn is None or not payload_len or not isinstance(header, dict):
            return None
        dtype, shape = header.get("dtype"), header.get("shape")
        if dtype not in WIRE_DTYPES or not isinstance(shape, list) or len(shape) > 16:
            return None
        if not all(isinstance(d, int) and not isinstance(d, bool) and d >= 0 for d in shape):
            return None
        tdt = WIRE_DTYPES[dtype]
        if math.prod(shape) * torch.empty((), dtype=tdt).element_size() != payload_len:
            return None
        buf = fn(header.get("message_type"), tdt, tuple(shape))
        if buf is None or buf.device.type != "cpu" or not buf.is_contiguous():
            return None
        if buf.numel() * buf.element_size() != payload_len:
            return None
        return buf

    @abc.abstractmethod
    def _send_frame(self, frame) -> None: ...

    def _send_parts(self, head: bytes, payload) -> None:
        self._send_frame(head + bytes(payload))

    @abc.abstractmethod
    def _recv_packet(self, timeout: float | None) -> tuple[TensorPacket, int]: ...

    @abc.abstractmethod
    def close(self) -> None: ...

    def send_packet(self, packet: TensorPacket) -> float:
        """Send one packet; returns the seconds spent sending."""
        if len(packet.payload) > self.max_payload_bytes:
            raise ProtocolError(f"payload {len(packet.payload)} exceeds limit {self.max_payload_bytes}")
        head = encode_head(packet)
        t0 = time.perf_counter()
        with self._send_lock:
            self._send_parts(head, packet.payload)
        self.bytes_sent += len(head) + len(packet.payload)
        return time.perf_counter() - t0

    def recv_packet(self, timeout: float | None = None) -> TensorPacket:
        packet, n = self._recv_packet(timeout)
        self.bytes_received += n
        return packet

    def send_tensor(self, tensor: torch.Tensor, message_type: MessageType, *, device=None,
                    lifecycle: TensorLifecycle | None = None, **fields) -> TensorLifecycle:
        lc = lifecycle if lifecycle is not None else TensorLifecycle()
        pkt = tensor_to_packet(tensor, message_type, device=device, lifecycle=lc, **fields)
        lc.add("network_send", self.send_packet(pkt))
        return lc

    def recv_tensor(self, timeout: float | None = None, *, device=None):
        lc = TensorLifecycle()
        t0 = time.perf_counter()
        pkt = self.recv_packet(timeout)
        lc.add("network_recv", time.perf_counter() - t0)
        return packet_to_tensor(pkt, device=device, lifecycle=lc), pkt


class PipeTransport(Transport):
    """Transport over a multiprocessing ``Connection`` (same host)."""

    def __init__(self, conn, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES):
        super().__init__(max_payload_bytes)
        self.conn = conn

    def _send_frame(self, frame) -> None:
        try:
            self.conn.send_bytes(frame)
        except (BrokenPipeError, OSError, EOFError) as exc:
            raise TransportClosed(f"peer closed pipe: {exc}") from exc

    def _recv_packet(self, timeout):
        try:
            ready = self.conn.poll(timeout)
        except (EOFError, BrokenPipeError, ConnectionResetError, OSError) as exc:
            raise TransportClosed(f"peer closed pipe: {exc}") from exc
        if not ready:
            raise TransportTimeout(f"no packet within {timeout}s")
        try:
            frame = self.conn.recv_bytes(PREFIX_SIZE + 64 * 1024 + self.max_payload_bytes)
        except (EOFError, BrokenPipeError, ConnectionResetError) as exc:
            raise TransportClosed(f"peer closed pipe: {exc}") from exc
        except OSError as exc:
            raise ProtocolError(f"pipe receive failed: {exc}") from exc
        return decode_packet(frame, self.max_payload_bytes), len(frame)

    def close(self) -> None:
        try:
            self.conn.close()
        except OSError:
            pass

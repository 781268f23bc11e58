"""Packet links between pipeline peers.

A link carries ``TensorPacket``s in order, reliably, in both directions, and
counts the bytes it moved.  It is made of two layers:

* an *endpoint* moves raw bytes.  ``ConnectionEndpoint`` wraps a
  multiprocessing ``Connection`` (stage processes on one host; each frame is one
  message) and ``SocketEndpoint`` (networking/tcp.py) a connected TCP socket
  (bytes are a stream).  Both offer the same three calls: ``wait(timeout)``,
  ``read_exact(n, into=None)`` and ``write(chunks)``.
* ``Transport`` speaks MSHT v1 (networking/protocol.py) over any endpoint: it
  cuts frames, validates them, can receive a payload straight into a buffer
  the caller supplies (``payload_allocator``), serialises concurrent senders
  and keeps the byte counters.

``PipeTransport`` and ``TCPTransport`` are ``Transport`` over the two
endpoints.  GPU stages inside one box do not use these links: they exchange
activations with NCCL (parallel/p2p.py).  Behaviour matches the reference's
links (networking/transport.py:52-170, networking/tcp.py:27-104): a receive
waits ``timeout`` for the *start* of a frame and then reads the whole frame.
"""

from __future__ import annotations

import math
import threading
import time

import torch

from meshtrain_b200.networking.packet import WIRE_DTYPES, MessageType, TensorPacket
from meshtrain_b200.networking.protocol import (
    DEFAULT_MAX_PAYLOAD_BYTES, MAX_HEADER_BYTES, PREFIX_SIZE, ProtocolError, encode_head, packet_from_header,
    parse_header, parse_prefix)
from meshtrain_b200.networking.serialization import TensorLifecycle, packet_to_tensor, tensor_to_packet


class TransportError(RuntimeError):
    pass


class TransportTimeout(TransportError, TimeoutError):
    pass


class TransportClosed(TransportError, ConnectionError):
    pass


def payload_buffer_for(allocator, header, payload_len: int):
    """The caller's receive buffer for a frame, or None to receive into fresh bytes.

    The header comes off the wire and is untrusted: a buffer is requested only
    for a well-formed tensor header whose dtype and shape account for exactly
    ``payload_len`` bytes, and used only if it is a contiguous CPU tensor of
    that size.
    """
    if allocator is None or payload_len == 0 or not isinstance(header, dict):
        return None
    dtype_name, shape = header.get("dtype"), header.get("shape")
    if dtype_name not in WIRE_DTYPES or not isinstance(shape, list) or len(shape) > 16:
        return None
    if any(isinstance(d, bool) or not isinstance(d, int) or d < 0 for d in shape):
        return None
    dtype = WIRE_DTYPES[dtype_name]
    if math.prod(shape) * dtype.itemsize != payload_len:
        return None
    buf = allocator(header.get("message_type"), dtype, tuple(shape))
    if not isinstance(buf, torch.Tensor) or buf.device.type != "cpu" or not buf.is_contiguous():
        return None
    return buf if buf.numel() * buf.element_size() == payload_len else None


class ConnectionEndpoint:
    """Bytes over a multiprocessing ``Connection``: one message per frame.

    ``read_exact`` serves reads from the current message and fetches the next
    message only when the current one is used up, so a frame never spans two
    messages.
    """

    def __init__(self, conn, max_message_bytes: int):
        self.conn = conn
        self.peer = "pipe"
        self.max_message_bytes = max_message_bytes
        self._msg = b""
        self._pos = 0

    def wait(self, timeout: float | None) -> bool:
        if self._pos < len(self._msg):
            return True
        try:
            return bool(self.conn.poll(timeout))
        except (EOFError, OSError) as exc:
            raise TransportClosed(f"peer closed pipe: {exc}") from exc

    def _next_message(self) -> None:
        try:
            self._msg = self.conn.recv_bytes(self.max_message_bytes)
        except (EOFError, BrokenPipeError, ConnectionResetError) as exc:
            raise TransportClosed(f"peer closed pipe: {exc}") from exc
        except OSError as exc:  # a message longer than the limit
            raise ProtocolError(f"pipe receive failed: {exc}") from exc
        self._pos = 0

    def read_exact(self, n: int, into: memoryview | None = None):
        if n and self._pos >= len(self._msg):
            self._next_message()
        if self._pos + n > len(self._msg):
            raise ProtocolError("frame is longer than the pipe message that carried it")
        chunk = memoryview(self._msg)[self._pos:self._pos + n]
        self._pos += n
        if into is None:
            return bytes(chunk)
        into[:n] = chunk
        return into

    def write(self, chunks) -> None:
        try:
            self.conn.send_bytes(b"".join(bytes(c) for c in chunks))
        except (BrokenPipeError, EOFError, OSError) as exc:
            raise TransportClosed(f"peer closed pipe: {exc}") from exc

    def close(self) -> None:
        try:
            self.conn.close()
        except OSError:
            pass


class PacketLink:
    """Tensor-level calls shared by every link type (built on send/recv_packet)."""

    def send_tensor(self, tensor: torch.Tensor, message_type: MessageType, *, device=None,
                    lifecycle: TensorLifecycle | None = None, **fields) -> TensorLifecycle:
        lc = TensorLifecycle() if lifecycle is None else lifecycle
        packet = tensor_to_packet(tensor, message_type, device=device, lifecycle=lc, **fields)
        lc.add("network_send", self.send_packet(packet))
        return lc

    def recv_tensor(self, timeout: float | None = None, *, device=None):
        lc = TensorLifecycle()
        t0 = time.perf_counter()
        packet = self.recv_packet(timeout)
        lc.add("network_recv", time.perf_counter() - t0)
        return packet_to_tensor(packet, device=device, lifecycle=lc), packet


class Transport(PacketLink):
    """MSHT v1 packets over an endpoint.

    ``payload_allocator(message_type, dtype, shape)`` may return a CPU tensor
    to receive a tensor payload into (the device layer's pinned pool); the
    packet then carries it as ``recv_buffer``.  ``last_frame_s`` is the time
    the last frame took on the wire once it had started.
    """

    def __init__(self, endpoint, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES):
        self.endpoint = endpoint
        self.max_payload_bytes = max_payload_bytes
        self.bytes_sent = 0
        self.bytes_received = 0
        self.last_frame_s = 0.0
        self.payload_allocator = None
        self._send_lock = threading.Lock()

    @property
    def peer(self) -> str:
        return self.endpoint.peer

    def send_packet(self, packet: TensorPacket) -> float:
        """Sends one packet; returns the seconds spent in the send."""
        size = len(packet.payload)
        if size > self.max_payload_bytes:
            raise ProtocolError(f"payload {size} exceeds limit {self.max_payload_bytes}")
        head = encode_head(packet)
        t0 = time.perf_counter()
        with self._send_lock:
            self.endpoint.write((head, packet.payload) if size else (head,))
            self.bytes_sent += len(head) + size
        return time.perf_counter() - t0

    def recv_packet(self, timeout: float | None = None) -> TensorPacket:
        if not self.endpoint.wait(timeout):
            raise TransportTimeout(f"no packet from {self.peer} within {timeout}s")
        t0 = time.perf_counter()
        read = self.endpoint.read_exact
        header_len, payload_len = parse_prefix(bytes(read(PREFIX_SIZE)), self.max_payload_bytes)
        header = parse_header(read(header_len))
        buf = payload_buffer_for(self.payload_allocator, header, payload_len)
        if buf is not None:
            read(payload_len, into=memoryview(buf.reshape(-1).view(torch.uint8).numpy()))
            payload = memoryview(buf.reshape(-1).view(torch.uint8).numpy())
        else:
            payload = read(payload_len) if payload_len else b""
        self.last_frame_s = time.perf_counter() - t0
        packet = packet_from_header(header, payload)
        packet.recv_buffer = buf
        self.bytes_received += PREFIX_SIZE + header_len + payload_len
        return packet

    def close(self) -> None:
        self.endpoint.close()


class PipeTransport(Transport):
    """A link over a multiprocessing ``Connection`` (stages as processes on one host)."""

    def __init__(self, conn, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES):
        super().__init__(ConnectionEndpoint(conn, PREFIX_SIZE + MAX_HEADER_BYTES + max_payload_bytes),
                         max_payload_bytes)

    @property
    def conn(self):
        return self.endpoint.conn

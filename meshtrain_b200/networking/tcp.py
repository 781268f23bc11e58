"""Raw-TCP data plane: one connection per pipeline link, MSHT frames both ways.

The connecting side first sends a CONTROL "HELLO" packet (job id, stage,
cluster token) so a worker's single listener can route connections
(reference networking/tcp.py:27-162).  Receives wait for the start of a frame
with a timeout, then read the whole frame (bounded by ``frame_timeout_s``),
optionally straight into a caller-provided tensor buffer.
"""

from __future__ import annotations

import select
import socket
import time

import torch

from meshtrain_b200.networking.packet import MessageType, TensorPacket
from meshtrain_b200.networking.protocol import (
    DEFAULT_MAX_PAYLOAD_BYTES, PREFIX_SIZE, ProtocolError, packet_from_header, parse_header, parse_prefix)
from meshtrain_b200.networking.transport import Transport, TransportClosed, TransportTimeout

_CHUNK = 4 * 1024 * 1024


def _recv_exact(sock: socket.socket, n: int, into: memoryview | None = None):
    buf = into if into is not None else bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        try:
            k = sock.recv_into(view[got:], min(n - got, _CHUNK))
        except socket.timeout as exc:
            raise TransportTimeout(f"peer stalled mid-frame ({got}/{n} bytes)") from exc
        except OSError as exc:
            raise TransportClosed(f"connection error: {exc}") from exc
        if k == 0:
            raise TransportClosed("peer closed the connection")
        got += k
    return buf


class TCPTransport(Transport):
    def __init__(self, sock: socket.socket, *, frame_timeout_s: float = 60.0,
                 max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES, peer: str = ""):
        super().__init__(max_payload_bytes)
        self.sock = sock
        self.frame_timeout_s = frame_timeout_s
        try:
            self.peer = peer or "%s:%s" % sock.getpeername()[:2]
        except OSError:
            self.peer = peer or "?"
        sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        sock.settimeout(frame_timeout_s)

    def _send_frame(self, frame) -> None:
        try:
            self.sock.sendall(frame)
        except socket.timeout as exc:
            raise TransportTimeout(f"send to {self.peer} timed out") from exc
        except OSError as exc:
            raise TransportClosed(f"send to {self.peer} failed: {exc}") from exc

    def _send_parts(self, head: bytes, payload) -> None:
        self._send_frame(head)
        if len(payload):
            self._send_frame(payload)  # zero-copy: the payload view goes straight to the socket

    def _recv_packet(self, timeout):
        try:
            ready, _, _ = select.select([self.sock], [], [], timeout)
        except (OSError, ValueError) as exc:
            raise TransportClosed(f"connection to {self.peer} closed: {exc}") from exc
        if not ready:
            raise TransportTimeout(f"no packet from {self.peer} within {timeout}s")
        t0 = time.perf_counter()
        prefix = _recv_exact(self.sock, PREFIX_SIZE)
        hlen, plen = parse_prefix(bytes(prefix), self.max_payload_bytes)
        header = parse_header(bytes(_recv_exact(self.sock, hlen)))
        target = self._allocate(header, plen)
        if target is not None:
            payload = _recv_exact(self.sock, plen, into=memoryview(target.reshape(-1).view(torch.uint8).numpy()))
        else:
            payload = _recv_exact(self.sock, plen) if plen else b""
        self.last_frame_s = time.perf_counter() - t0
        pkt = packet_from_header(header, payload)
        pkt.recv_buffer = target
        return pkt, PREFIX_SIZE + hlen + plen

    def close(self) -> None:
        try:
            self.sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self.sock.close()


def hello_packet(hello: dict) -> TensorPacket:
    return TensorPacket(MessageType.CONTROL, job_id=str(hello.get("job_id", "")), meta={"command": "HELLO", **hello})


def connect(host: str, port: int, *, timeout: float = 30.0, hello: dict | None = None, frame_timeout_s: float = 60.0,
            max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES, stop_event=None) -> TCPTransport:
    """Connect, retrying until ``timeout`` (the peer may still be starting), then send HELLO."""
    deadline = time.monotonic() + timeout
    last: Exception | None = None
    while time.monotonic() < deadline:
        if stop_event is not None and stop_event.is_set():
            raise TransportTimeout("connect cancelled: job stopped")
        try:
            sock = socket.create_connection((host, port), timeout=min(5.0, timeout))
            break
        except OSError as exc:
            last = exc
            time.sleep(0.1)
    else:
        raise TransportTimeout(f"could not connect to {host}:{port} within {timeout}s: {last}")
    t = TCPTransport(sock, frame_timeout_s=frame_timeout_s, max_payload_bytes=max_payload_bytes, peer=f"{host}:{port}")
    t.send_packet(hello_packet(hello or {}))
    return t


class TCPListener:
    def __init__(self, host: str = "0.0.0.0", port: int = 0, *, token: str | None = None,
                 frame_timeout_s: float = 60.0, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES):
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.sock.bind((host, port))
        self.sock.listen(16)
        self.port = self.sock.getsockname()[1]
        self.token = token
        self.frame_timeout_s = frame_timeout_s
        self.max_payload_bytes = max_payload_bytes

    def accept(self, timeout: float | None = None) -> tuple[TCPTransport, dict]:
        """Accept one connection and validate its HELLO (and token)."""
        self.sock.settimeout(timeout)
        try:
            conn, addr = self.sock.accept()
        except socket.timeout as exc:
            raise TransportTimeout(f"no peer connected within {timeout}s") from exc
        t = TCPTransport(conn, frame_timeout_s=self.frame_timeout_s, max_payload_bytes=self.max_payload_bytes,
                         peer=f"{addr[0]}:{addr[1]}")
        try:
            hello = t.recv_packet(timeout=min(timeout or 10.0, 10.0))
            if hello.message_type != MessageType.CONTROL or hello.meta.get("command") != "HELLO":
                raise ProtocolError("first packet must be a HELLO control packet")
            if self.token is not None and hello.meta.get("token") != self.token:
                raise ProtocolError("invalid cluster token")
        except Exception:
            t.close()
            raise
        return t, dict(hello.meta)

    def close(self) -> None:
        self.sock.close()

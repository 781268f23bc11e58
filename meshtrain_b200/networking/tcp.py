"""Raw-TCP data plane: one connection per pipeline link, MSHT frames both ways.

A worker has one listening socket for all of its links, so the dialling side
opens every connection with a CONTROL packet whose ``meta.command`` is
``HELLO`` (job id, stage, cluster token); the accepting side checks it before
the link is used.  Same handshake and wire behaviour as the reference
(networking/tcp.py:27-162): a receive waits for the start of a frame with the
caller's timeout, then reads the whole frame within ``frame_timeout_s``,
optionally straight into a caller-provided tensor.
"""

from __future__ import annotations

import select
import socket
import time

from meshtrain_b200.networking.packet import MessageType, TensorPacket
from meshtrain_b200.networking.protocol import DEFAULT_MAX_PAYLOAD_BYTES, ProtocolError
from meshtrain_b200.networking.transport import Transport, TransportClosed, TransportTimeout

# Largest single recv_into; bounds the time one call can block inside a frame.
_RECV_SLICE = 4 << 20


class SocketEndpoint:
    """Bytes over a connected stream socket (TCP_NODELAY, per-call timeouts)."""

    def __init__(self, sock: socket.socket, frame_timeout_s: float, peer: str = ""):
        self.sock = sock
        if not peer:
            try:
                host, port = sock.getpeername()[:2]
                peer = f"{host}:{port}"
            except OSError:
                peer = "?"
        self.peer = peer
        sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        sock.settimeout(frame_timeout_s)

    def wait(self, timeout: float | None) -> bool:
        try:
            readable, _, _ = select.select([self.sock], [], [], timeout)
        except (OSError, ValueError) as exc:  # closed under us
            raise TransportClosed(f"connection to {self.peer} closed: {exc}") from exc
        return bool(readable)

    def read_exact(self, n: int, into: memoryview | None = None):
        out = bytearray(n) if into is None else into
        view = memoryview(out)
        done = 0
        while done < n:
            try:
                got = self.sock.recv_into(view[done:], min(n - done, _RECV_SLICE))
            except socket.timeout as exc:
                raise TransportTimeout(f"{self.peer} stalled mid-frame after {done} of {n} bytes") from exc
            except OSError as exc:
                raise TransportClosed(f"connection to {self.peer} failed: {exc}") from exc
            if got == 0:
                raise TransportClosed(f"{self.peer} closed the connection")
            done += got
        return out

    def write(self, chunks) -> None:
        # header and payload go out as separate sendall calls: the payload view
        # reaches the socket without being copied into one frame buffer
        try:
            for chunk in chunks:
                self.sock.sendall(chunk)
        except socket.timeout as exc:
            raise TransportTimeout(f"send to {self.peer} timed out") from exc
        except OSError as exc:
            raise TransportClosed(f"send to {self.peer} failed: {exc}") from exc

    def close(self) -> None:
        try:
            self.sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self.sock.close()


class TCPTransport(Transport):
    """A link over one TCP connection."""

    def __init__(self, sock: socket.socket, *, frame_timeout_s: float = 60.0,
                 max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES, peer: str = ""):
        super().__init__(SocketEndpoint(sock, frame_timeout_s, peer), max_payload_bytes)
        self.frame_timeout_s = frame_timeout_s

    @property
    def sock(self) -> socket.socket:
        return self.endpoint.sock


def hello_packet(hello: dict) -> TensorPacket:
    """The first packet on every data-plane connection."""
    return TensorPacket(MessageType.CONTROL, job_id=str(hello.get("job_id", "")), meta={"command": "HELLO", **hello})


def _dial(host: str, port: int, timeout: float, stop_event) -> socket.socket:
    """Connects, retrying every 0.1 s until ``timeout``: the peer may still be starting."""
    give_up = time.monotonic() + timeout
    error: Exception | None = None
    while True:
        if stop_event is not None and stop_event.is_set():
            raise TransportTimeout("connect cancelled: job stopped")
        left = give_up - time.monotonic()
        if left <= 0:
            raise TransportTimeout(f"could not connect to {host}:{port} within {timeout}s: {error}")
        try:
            return socket.create_connection((host, port), timeout=min(5.0, left))
        except OSError as exc:
            error = exc
            time.sleep(min(0.1, max(0.0, give_up - time.monotonic())))


def connect(host: str, port: int, *, timeout: float = 30.0, hello: dict | None = None, frame_timeout_s: float = 60.0,
            max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES, stop_event=None) -> TCPTransport:
    """Opens a link to ``host:port`` and sends the HELLO handshake."""
    link = TCPTransport(_dial(host, port, timeout, stop_event), frame_timeout_s=frame_timeout_s,
                        max_payload_bytes=max_payload_bytes, peer=f"{host}:{port}")
    link.send_packet(hello_packet(hello or {}))
    return link


def check_hello(packet: TensorPacket, token: str | None) -> dict:
    """Validates a HELLO packet (and the cluster token when one is required)."""
    if packet.message_type != MessageType.CONTROL or packet.meta.get("command") != "HELLO":
        raise ProtocolError("first packet must be a HELLO control packet")
    if token is not None and packet.meta.get("token") != token:
        raise ProtocolError("invalid cluster token")
    return dict(packet.meta)


class TCPListener:
    """A listening socket that hands out validated links."""

    def __init__(self, host: str = "0.0.0.0", port: int = 0, *, token: str | None = None,
                 frame_timeout_s: float = 60.0, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES):
        self.token = token
        self.frame_timeout_s = frame_timeout_s
        self.max_payload_bytes = max_payload_bytes
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.sock.bind((host, port))
        self.sock.listen(16)
        self.port = self.sock.getsockname()[1]

    def accept(self, timeout: float | None = None) -> tuple[TCPTransport, dict]:
        """Waits for one connection and returns it with its HELLO fields."""
        self.sock.settimeout(timeout)
        try:
            conn, (host, port) = self.sock.accept()[:2]
        except socket.timeout as exc:
            raise TransportTimeout(f"no peer connected within {timeout}s") from exc
        link = TCPTransport(conn, frame_timeout_s=self.frame_timeout_s, max_payload_bytes=self.max_payload_bytes,
                            peer=f"{host}:{port}")
        try:
            hello = check_hello(link.recv_packet(timeout=min(timeout or 10.0, 10.0)), self.token)
        except Exception:
            link.close()
            raise
        return link, hello

    def close(self) -> None:
        self.sock.close()

import multiprocessing as mp
import threading
import time

import pytest
import torch

from meshtrain_b200.networking.emulation import EmulatedLink
from meshtrain_b200.networking.packet import MessageType
from meshtrain_b200.networking.protocol import ProtocolError
from meshtrain_b200.networking.tcp import TCPListener, connect
from meshtrain_b200.networking.transport import PipeTransport, TransportClosed, TransportTimeout


def _tcp_pair(token=None, hello=None):
    lis = TCPListener("127.0.0.1", 0, token=token)
    box = {}

    def acc():
        try:
            box["server"] = lis.accept(timeout=10)
        except Exception as exc:  # noqa: BLE001
            box["error"] = exc

    t = threading.Thread(target=acc)
    t.start()
    client = connect("127.0.0.1", lis.port, timeout=10, hello=hello or {"job_id": "j"})
    t.join()
    lis.close()
    if "error" in box:
        client.close()
        raise box["error"]
    return client, *box["server"]


def test_tcp_roundtrip_and_hello():
    client, server, hello = _tcp_pair(hello={"job_id": "j1", "stage": 3})
    assert hello["stage"] == 3 and hello["job_id"] == "j1"
    x = torch.randn(64, 33)
    client.send_tensor(x, MessageType.FORWARD_ACTIVATION, step_id=4, microbatch_id=2)
    pkt_t, pkt = server.recv_tensor(timeout=5)
    assert torch.equal(pkt_t, x) and pkt.step_id == 4 and pkt.microbatch_id == 2
    server.send_tensor(x * 2, MessageType.BACKWARD_GRADIENT)
    back, _ = client.recv_tensor(timeout=5)
    assert torch.equal(back, x * 2)
    assert client.bytes_sent > x.numel() * 4 and server.bytes_received > x.numel() * 4
    client.close()
    server.close()


def test_tcp_token_is_checked():
    with pytest.raises(ProtocolError, match="token"):
        _tcp_pair(token="secret", hello={"job_id": "j", "token": "wrong"})
    c, s, h = _tcp_pair(token="secret", hello={"job_id": "j", "token": "secret"})
    c.close()
    s.close()


def test_tcp_recv_timeout_and_peer_close():
    client, server, _ = _tcp_pair()
    with pytest.raises(TransportTimeout):
        server.recv_packet(timeout=0.2)
    client.close()
    with pytest.raises((TransportClosed, ConnectionError)):
        server.recv_packet(timeout=2)
    server.close()


def test_connect_timeout_when_nobody_listens():
    lis = TCPListener("127.0.0.1", 0)
    port = lis.port
    lis.close()
    with pytest.raises(TransportTimeout):
        connect("127.0.0.1", port, timeout=0.5)


def test_pipe_transport_roundtrip():
    a, b = mp.Pipe(duplex=True)
    ta, tb = PipeTransport(a), PipeTransport(b)
    x = torch.randn(10, 10, dtype=torch.float64)
    ta.send_tensor(x, MessageType.FORWARD_ACTIVATION, step_id=1)
    got, pkt = tb.recv_tensor(timeout=2)
    assert torch.equal(got, x) and pkt.step_id == 1
    with pytest.raises(TransportTimeout):
        tb.recv_packet(timeout=0.1)
    ta.close()
    tb.close()


def test_emulated_link_throttles_bandwidth():
    a, b = mp.Pipe(duplex=True)
    slow = EmulatedLink(PipeTransport(a), bandwidth_bytes_per_s=4e6, latency_s=0.01)
    rx = PipeTransport(b)
    x = torch.zeros(100_000)  # 400 kB -> ~0.1 s at 4 MB/s
    got = {}
    reader = threading.Thread(target=lambda: got.update(t=rx.recv_tensor(timeout=5)[0]))
    reader.start()  # a pipe holds ~64 kB: the reader must drain it while the sender writes
    t0 = time.perf_counter()
    slow.send_tensor(x, MessageType.FORWARD_ACTIVATION)
    reader.join()
    assert torch.equal(got["t"], x)
    assert time.perf_counter() - t0 >= 0.09
    assert slow.wire_time(4_000_000) == pytest.approx(1.01, rel=1e-6)
    slow.close()
    rx.close()

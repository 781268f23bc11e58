"""Directional link probes between workers, plus an NCCL probe between GPUs of one box.

TCP probe protocol (a connection opened with a HELLO whose ``command_kind`` is
``PROBE``; the same messages as the reference's probe, profiler/network.py:26-88,
so either side can be a reference worker):

    prober                              served side
    CONTROL {op: PING}          ->      ACK {op: PONG}          (repeated: round-trip time)
    FORWARD_ACTIVATION blobs    ->      counted, no reply       (bulk transfer)
    CONTROL {op: SYNC}          ->      ACK {bytes: n}          (bytes counted since the last SYNC)
    CONTROL {op: BYE}           ->      connection done

The link's one-way latency is half the median round trip; its bandwidth is the
bytes acknowledged at SYNC over the bulk phase's time minus one round trip.
``measure_nccl_link`` times device-to-device sends between two ranks with CUDA
events.
"""

from __future__ import annotations

import statistics
import time

import torch

from meshtrain_b200.networking.packet import MessageType, TensorPacket
from meshtrain_b200.networking.tcp import connect


def _control(op: str) -> TensorPacket:
    return TensorPacket(MessageType.CONTROL, meta={"op": op})


class ProbeSession:
    """Served side of one probe connection."""

    def __init__(self, link):
        self.link = link
        self.counted = 0
        self.open = True

    def on_ping(self, _packet) -> None:
        self.link.send_packet(TensorPacket(MessageType.ACK, meta={"op": "PONG"}))

    def on_sync(self, _packet) -> None:
        self.link.send_packet(TensorPacket(MessageType.ACK, meta={"bytes": self.counted}))
        self.counted = 0

    def on_bye(self, _packet) -> None:
        self.open = False

    HANDLERS = {"PING": on_ping, "SYNC": on_sync, "BYE": on_bye}

    def run(self, timeout: float) -> None:
        while self.open:
            packet = self.link.recv_packet(timeout=timeout)
            if packet.message_type == MessageType.CONTROL:
                handler = self.HANDLERS.get(packet.meta.get("op"))
                if handler is not None:
                    handler(self, packet)
            elif packet.has_tensor:
                self.counted += len(packet.payload)


def serve_probe(link, timeout: float = 30.0) -> None:
    """Answers a prober on ``link`` until it says BYE."""
    ProbeSession(link).run(timeout)


def measure_link(host: str, port: int, *, token: str | None = None, pings: int = 10, payload_mb: float = 16.0,
                 chunks: int = 4, timeout: float = 30.0) -> dict:
    """Latency and bandwidth from this host to the worker listening at host:port."""
    hello = {"probe": True, "command_kind": "PROBE", **({"token": token} if token is not None else {})}
    link = connect(host, port, timeout=timeout, hello=hello, frame_timeout_s=timeout)
    try:
        round_trips = []
        for _ in range(pings):
            sent = time.perf_counter()
            link.send_packet(_control("PING"))
            link.recv_packet(timeout=timeout)
            round_trips.append(time.perf_counter() - sent)
        blob = torch.zeros(max(1, int(payload_mb * 1e6 / 4 / chunks)))
        began = time.perf_counter()
        for _ in range(chunks):
            link.send_tensor(blob, MessageType.FORWARD_ACTIVATION)
        link.send_packet(_control("SYNC"))
        acked = int(link.recv_packet(timeout=timeout).meta.get("bytes", 0))
        bulk_s = time.perf_counter() - began
        link.send_packet(_control("BYE"))
    finally:
        link.close()
    rtt = statistics.median(round_trips)
    wire_s = max(bulk_s - rtt, 1e-9)
    return {"latency_s": rtt / 2, "rtt_s": rtt, "bandwidth_Bps": acked / wire_s,
            "bandwidth_Mbps": acked * 8 / wire_s / 1e6, "bytes": acked, "kind": "tcp"}


def measure_nccl_link(src: int, dst: int, *, nbytes: int = 32 * 1024 ** 2, iters: int = 10, group=None) -> dict | None:
    """Times ``src`` -> ``dst`` NCCL sends (every rank of ``group`` calls it); the result is on ``src``."""
    import torch.distributed as dist

    rank = dist.get_rank()
    if rank not in (src, dst):
        return None
    buf = torch.zeros(nbytes // 2, dtype=torch.bfloat16, device=torch.device("cuda", torch.cuda.current_device()))
    seconds = []
    for _ in range(iters + 2):  # the first two warm the connection up
        if rank == dst:
            dist.recv(buf, src, group=group)
            torch.cuda.synchronize()
            continue
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        dist.send(buf, dst, group=group)
        end.record()
        end.synchronize()
        seconds.append(start.elapsed_time(end) / 1e3)
    if rank == dst:
        return None
    best = min(seconds[2:])
    return {"latency_s": 10e-6, "bandwidth_Bps": nbytes / best, "bandwidth_Mbps": nbytes * 8 / best / 1e6,
            "bytes": nbytes, "seconds": best, "kind": "nccl"}


def format_matrix(names: list[str], values: dict[tuple[str, str], float], fmt) -> str:
    """Square text table of a per-pair quantity (rows: source, columns: destination)."""
    width = max([10] + [len(n) + 2 for n in names])
    rows = [" " * width + "".join(n.rjust(width) for n in names)]
    for src in names:
        cells = ("-" if src == dst else fmt(values.get((src, dst))) for dst in names)
        rows.append(src.ljust(width) + "".join(str(c).rjust(width) for c in cells))
    return "\n".join(rows)

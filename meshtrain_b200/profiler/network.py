"""Directional link probes (reference profiler/network.py:26-88) plus an NCCL p2p probe.

TCP probe, after a HELLO with ``command=PROBE``:
    client: CONTROL{op=PING}            server: ACK
    client: FORWARD_ACTIVATION blob xN  (no reply)
    client: CONTROL{op=SYNC}            server: ACK{bytes}
    client: CONTROL{op=BYE}
bandwidth = bytes / (elapsed - RTT).  ``measure_nccl_link`` times a device-to-
device send between two ranks of one box with CUDA events.
"""

from __future__ import annotations

import statistics
import time

import torch

from meshtrain_b200.networking.packet import MessageType, TensorPacket
from meshtrain_b200.networking.tcp import connect


def serve_probe(link, timeout: float = 30.0) -> None:
    received = 0
    while True:
        p = link.recv_packet(timeout=timeout)
        if p.message_type == MessageType.CONTROL:
            op = p.meta.get("op")
            if op == "PING":
                link.send_packet(TensorPacket(MessageType.ACK, meta={"op": "PONG"}))
            elif op == "SYNC":
                link.send_packet(TensorPacket(MessageType.ACK, meta={"bytes": received}))
                received = 0
            elif op == "BYE":
                return
        elif p.has_tensor:
            received += len(p.payload)


def measure_link(host: str, port: int, *, token: str | None = None, pings: int = 10, payload_mb: float = 16.0,
                 chunks: int = 4, timeout: float = 30.0) -> dict:
    hello = {"probe": True, "command_kind": "PROBE"}
    if token is not None:
        hello["token"] = token
    link = connect(host, port, timeout=timeout, hello=hello, frame_timeout_s=timeout)
    try:
        rtts = []
        for _ in range(pings):
            t0 = time.perf_counter()
            link.send_packet(TensorPacket(MessageType.CONTROL, meta={"op": "PING"}))
            link.recv_packet(timeout=timeout)
            rtts.append(time.perf_counter() - t0)
        blob = torch.zeros(max(1, int(payload_mb * 1e6 / 4 / chunks)))
        t0 = time.perf_counter()
        for _ in range(chunks):
            link.send_tensor(blob, MessageType.FORWARD_ACTIVATION)
        link.send_packet(TensorPacket(MessageType.CONTROL, meta={"op": "SYNC"}))
        ack = link.recv_packet(timeout=timeout)
        elapsed = time.perf_counter() - t0
        nbytes = int(ack.meta.get("bytes", 0))
        link.send_packet(TensorPacket(MessageType.CONTROL, meta={"op": "BYE"}))
    finally:
        link.close()
    rtt = statistics.median(rtts)
    transfer = max(elapsed - rtt, 1e-9)
    return {"latency_s": rtt / 2, "rtt_s": rtt, "bandwidth_Bps": nbytes / transfer,
            "bandwidth_Mbps": nbytes * 8 / transfer / 1e6, "bytes": nbytes, "kind": "tcp"}


def measure_nccl_link(src: int, dst: int, *, nbytes: int = 32 * 1024 ** 2, iters: int = 10, group=None) -> dict | None:
    """Time ``src`` -> ``dst`` NCCL sends (call on every rank of ``group``); result on ``src``."""
    import torch.distributed as dist

    rank = dist.get_rank()
    if rank not in (src, dst):
        return None
    dev = torch.device("cuda", torch.cuda.current_device())
    buf = torch.zeros(nbytes // 2, dtype=torch.bfloat16, device=dev)
    times = []
    for _ in range(iters + 2):
        if rank == src:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            dist.send(buf, dst, group=group)
            e.record()
            e.synchronize()
            times.append(s.elapsed_time(e) / 1e3)
        else:
            dist.recv(buf, src, group=group)
            torch.cuda.synchronize(dev)
    if rank != src:
        return None
    t = min(times[2:])
    return {"latency_s": 10e-6, "bandwidth_Bps": nbytes / t, "bandwidth_Mbps": nbytes * 8 / t / 1e6, "bytes": nbytes,
            "seconds": t, "kind": "nccl"}


def format_matrix(names: list[str], values: dict[tuple[str, str], float], fmt) -> str:
    width = max(10, *(len(n) + 2 for n in names))
    lines = [" " * width + "".join(f"{n:>{width}}" for n in names)]
    for i in names:
        row = f"{i:<{width}}"
        for j in names:
            row += f"{'-':>{width}}" if i == j else f"{fmt(values.get((i, j))):>{width}}"
        lines.append(row)
    return "\n".join(lines)

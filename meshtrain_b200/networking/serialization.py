"""CPU tensor <-> packet conversion with per-phase timing.

``TensorLifecycle`` records how long each phase of moving one tensor took
(detach, to_cpu, serialize, network, deserialize, to_device), which feeds the
timeline and the communication breakdown (reference runtime/serialization.py:27-121).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from meshtrain_b200.networking.packet import DTYPE_NAMES, WIRE_DTYPES, MessageType, TensorPacket

PHASES = ("detach", "to_cpu", "serialize", "network_send", "network_recv", "deserialize", "to_device")


@dataclass
class TensorLifecycle:
    seconds: dict[str, float] = field(default_factory=dict)

    def add(self, phase: str, dt: float) -> None:
        self.seconds[phase] = self.seconds.get(phase, 0.0) + dt

    def total(self) -> float:
        return sum(self.seconds.values())


def tensor_to_bytes(t: torch.Tensor, copy: bool = True):
    """C-contiguous bytes of a CPU tensor (a memoryview when ``copy`` is False)."""
    if t.device.type != "cpu":
        raise ValueError("tensor_to_bytes needs a CPU tensor")
    t = t.contiguous()
    if t.numel() == 0:
        return b""
    raw = t.reshape(-1).view(torch.uint8)
    mv = memoryview(raw.numpy()).cast("B")
    return bytes(mv) if copy else mv


def bytes_to_tensor(data, dtype_name: str, shape) -> torch.Tensor:
    dtype = WIRE_DTYPES[dtype_name]
    shape = tuple(shape)
    if len(data) == 0:
        return torch.empty(shape, dtype=dtype)
    flat = torch.frombuffer(bytearray(data), dtype=torch.uint8)
    return flat.view(dtype).reshape(shape)


def tensor_to_packet(tensor: torch.Tensor, message_type: MessageType, *, device=None,
                     lifecycle: TensorLifecycle | None = None, copy: bool = True, **fields) -> TensorPacket:
    lc = lifecycle if lifecycle is not None else TensorLifecycle()
    t0 = time.perf_counter()
    t = tensor.detach()
    lc.add("detach", time.perf_counter() - t0)
    t0 = time.perf_counter()
    t = device.to_host(t) if device is not None and hasattr(device, "to_host") else t.cpu()
    lc.add("to_cpu", time.perf_counter() - t0)
    if t.dtype not in DTYPE_NAMES:
        raise TypeError(f"dtype {t.dtype} cannot be sent")
    t0 = time.perf_counter()
    payload = tensor_to_bytes(t, copy=copy)
    lc.add("serialize", time.perf_counter() - t0)
    return TensorPacket(message_type, shape=tuple(t.shape), dtype=DTYPE_NAMES[t.dtype], payload=payload, **fields)


def packet_to_tensor(packet: TensorPacket, *, device=None, lifecycle: TensorLifecycle | None = None) -> torch.Tensor:
    if not packet.has_tensor:
        raise ValueError("packet carries no tensor")
    lc = lifecycle if lifecycle is not None else TensorLifecycle()
    t0 = time.perf_counter()
    t = bytes_to_tensor(packet.payload, packet.dtype, packet.shape)
    lc.add("deserialize", time.perf_counter() - t0)
    if device is not None:
        t0 = time.perf_counter()
        t = device.move_tensor(t) if hasattr(device, "move_tensor") else t.to(device)
        lc.add("to_device", time.perf_counter() - t0)
    return t

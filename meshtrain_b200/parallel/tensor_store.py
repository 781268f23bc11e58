"""Stable tensor identities and a tiered tensor store.

IDs: ``model.layers.<g>.<name>`` (+ ``.grad`` / ``.optim.<key>``) and
``act.s<step>.mb<m>.stage<s>.<kind>`` - identical whichever rank owns the layer
(reference runtime/tensor_store.py:31-149).  Unlike the reference, whose
``evict`` refuses, this store implements the host-RAM tier: a tensor can be
evicted from the accelerator to pinned host memory and prefetched back with an
asynchronous copy on a side stream.
"""

from __future__ import annotations

import abc
import enum
import threading
from dataclasses import dataclass

import torch


class MemoryTier(enum.Enum):
    LOCAL_ACCELERATOR = "local_accelerator"
    LOCAL_RAM = "local_ram"
    REMOTE_ACCELERATOR = "remote_accelerator"
    REMOTE_RAM = "remote_ram"
    LOCAL_NVME = "local_nvme"
    REMOTE_NVME = "remote_nvme"
    RECOMPUTE = "recompute"


class TensorRole(enum.Enum):
    PARAMETER = "parameter"
    GRADIENT = "gradient"
    OPTIMIZER_STATE = "optimizer_state"
    ACTIVATION = "activation"
    ACTIVATION_GRADIENT = "activation_gradient"


@dataclass
class TensorMeta:
    tensor_id: str
    owner: str
    shape: tuple[int, ...]
    dtype: str
    bytes: int
    role: TensorRole
    tier: MemoryTier

    def to_dict(self) -> dict:
        return {"tensor_id": self.tensor_id, "owner": self.owner, "shape": list(self.shape), "dtype": self.dtype,
                "bytes": self.bytes, "role": self.role.value, "tier": self.tier.value}


def parameter_id(layer_index: int, param_name: str) -> str:
    return f"model.layers.{layer_index}.{param_name}"


def activation_id(step: int, microbatch: int, stage: int, kind: str = "input") -> str:
    return f"act.s{step}.mb{microbatch}.stage{stage}.{kind}"


class TensorStore(abc.ABC):
    @abc.abstractmethod
    def put(self, tensor_id: str, tensor: torch.Tensor, role: TensorRole, tier: MemoryTier | None = None) -> TensorMeta: ...

    @abc.abstractmethod
    def get(self, tensor_id: str) -> torch.Tensor: ...

    @abc.abstractmethod
    def locate(self, tensor_id: str) -> TensorMeta: ...

    @abc.abstractmethod
    def evict(self, tensor_id: str, to: MemoryTier) -> None: ...

    @abc.abstractmethod
    def prefetch(self, tensor_id: str) -> None: ...


_LOCAL = (MemoryTier.LOCAL_ACCELERATOR, MemoryTier.LOCAL_RAM)


class LocalTensorStore(TensorStore):
    """Tensors owned by one stage; moves them between the accelerator and pinned host RAM."""

    def __init__(self, owner: str, device_type: str = "cpu", device: torch.device | None = None):
        self.owner = owner
        self.home = MemoryTier.LOCAL_RAM if device_type == "cpu" else MemoryTier.LOCAL_ACCELERATOR
        self.device = device
        self._tensors: dict[str, torch.Tensor] = {}
        self._meta: dict[str, TensorMeta] = {}
        self._homes: dict[str, torch.device] = {}
        self._inflight: dict[str, object] = {}
        self._lock = threading.Lock()
        self._stream = None

    @staticmethod
    def _dtype_name(t: torch.Tensor) -> str:
        return str(t.dtype).replace("torch.", "")

    def put(self, tensor_id, tensor, role, tier=None):
        tier = tier or (MemoryTier.LOCAL_RAM if tensor.device.type == "cpu" else MemoryTier.LOCAL_ACCELERATOR)
        if tier not in _LOCAL:
            raise NotImplementedError(f"{tier.value} is not a tier this store can hold")
        meta = TensorMeta(tensor_id, self.owner, tuple(tensor.shape), self._dtype_name(tensor),
                          tensor.numel() * tensor.element_size(), role, tier)
        with self._lock:
            self._tensors[tensor_id] = tensor
            self._meta[tensor_id] = meta
            self._homes.setdefault(tensor_id, tensor.device)
        return meta

    def discard(self, tensor_id: str) -> None:
        with self._lock:
            self._tensors.pop(tensor_id, None)
            self._meta.pop(tensor_id, None)
            self._homes.pop(tensor_id, None)
            self._inflight.pop(tensor_id, None)

    def get(self, tensor_id):
        with self._lock:
            ev = self._inflight.pop(tensor_id, None)
            try:
                t = self._tensors[tensor_id]
            except KeyError:
                raise KeyError(f"tensor {tensor_id!r} is not owned by {self.owner}") from None
        if ev is not None and t.is_cuda:
            torch.cuda.current_stream(t.device).wait_event(ev)
        return t

    def locate(self, tensor_id):
        try:
            return self._meta[tensor_id]
        except KeyError:
            raise KeyError(f"tensor {tensor_id!r} is not owned by {self.owner}") from None

    def _side_stream(self, dev: torch.device):
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=dev)
        return self._stream

    def evict(self, tensor_id, to):
        """Move a tensor to pinned host RAM (the only non-resident tier implemented here)."""
        if to is not MemoryTier.LOCAL_RAM:
            raise NotImplementedError(f"eviction to {to.value} is not implemented")
        meta = self.locate(tensor_id)
        if meta.tier is MemoryTier.LOCAL_RAM:
            return
        t = self.get(tensor_id)
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=torch.cuda.is_available())
        host.copy_(t, non_blocking=False)
        with self._lock:
            self._tensors[tensor_id] = host
            meta.tier = MemoryTier.LOCAL_RAM

    def prefetch(self, tensor_id):
        """Start copying an evicted tensor back to its accelerator (async, side stream)."""
        meta = self.locate(tensor_id)
        home = self._homes.get(tensor_id)
        if meta.tier is not MemoryTier.LOCAL_RAM or home is None or home.type != "cuda":
            return
        host = self._tensors[tensor_id]
        stream = self._side_stream(home)
        with torch.cuda.stream(stream):
            dev = host.to(home, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
        with self._lock:
            self._tensors[tensor_id] = dev
            self._inflight[tensor_id] = ev
            meta.tier = MemoryTier.LOCAL_ACCELERATOR

    def ids(self, role: TensorRole | None = None) -> list[str]:
        with self._lock:
            return sorted(k for k, m in self._meta.items() if role is None or m.role is role)

    def bytes_by_role(self) -> dict[str, int]:
        out = {r.value: 0 for r in TensorRole}
        with self._lock:
            for m in self._meta.values():
                out[m.role.value] += m.bytes
        return out

    def bytes_by_tier(self) -> dict[str, int]:
        out: dict[str, int] = {}
        with self._lock:
            for m in self._meta.values():
                out[m.tier.value] = out.get(m.tier.value, 0) + m.bytes
        return out

    def manifest(self) -> list[dict]:
        with self._lock:
            return [self._meta[k].to_dict() for k in sorted(self._meta)]

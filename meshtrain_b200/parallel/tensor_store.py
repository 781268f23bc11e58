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
import dataclasses
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
        """JSON form used in stage manifests: enums as their values, the shape as a list."""
        row = dataclasses.asdict(self)
        row.update(shape=list(self.shape), role=self.role.value, tier=self.tier.value)
        return row


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


_HELD_HERE = (MemoryTier.LOCAL_ACCELERATOR, MemoryTier.LOCAL_RAM)


@dataclass
class _Entry:
    """One owned tensor: where it lives now, where it belongs, and a pending copy back."""

    tensor: torch.Tensor
    meta: TensorMeta
    home: torch.device
    ready: object = None  # CUDA event of an in-flight prefetch; consumers wait on it


class LocalTensorStore(TensorStore):
    """Tensors owned by one stage; moves them between the accelerator and pinned host RAM.

    Every tensor is one ``_Entry`` in a single table guarded by one lock.  Eviction
    copies to pinned host memory synchronously; prefetch copies back on a private
    side stream and records an event that the next ``get`` makes the caller's
    current stream wait on, so the copy overlaps whatever runs before that use.
    """

    def __init__(self, owner: str, device_type: str = "cpu", device: torch.device | None = None):
        self.owner = owner
        self.home = MemoryTier.LOCAL_RAM if device_type == "cpu" else MemoryTier.LOCAL_ACCELERATOR
        self.device = device
        self._table: dict[str, _Entry] = {}
        self._mu = threading.Lock()
        self._copy_stream = None

    def _find(self, tensor_id: str) -> _Entry:
        entry = self._table.get(tensor_id)
        if entry is None:
            raise KeyError(f"tensor {tensor_id!r} is not owned by {self.owner}")
        return entry

    def put(self, tensor_id, tensor, role, tier=None):
        natural = MemoryTier.LOCAL_RAM if tensor.device.type == "cpu" else MemoryTier.LOCAL_ACCELERATOR
        tier = tier or natural
        if tier not in _HELD_HERE:
            raise NotImplementedError(f"{tier.value} is not a tier this store can hold")
        meta = TensorMeta(tensor_id=tensor_id, owner=self.owner, shape=tuple(tensor.shape),
                          dtype=str(tensor.dtype).rsplit(".", 1)[-1], bytes=tensor.nbytes, role=role, tier=tier)
        with self._mu:
            old = self._table.get(tensor_id)
            # re-registering (a fresh gradient, a new optimizer state) keeps the original home device
            self._table[tensor_id] = _Entry(tensor, meta, old.home if old else tensor.device)
        return meta

    def discard(self, tensor_id: str) -> None:
        with self._mu:
            self._table.pop(tensor_id, None)

    def get(self, tensor_id):
        with self._mu:
            entry = self._find(tensor_id)
            pending, entry.ready = entry.ready, None
            tensor = entry.tensor
        if pending is not None and tensor.is_cuda:
            torch.cuda.current_stream(tensor.device).wait_event(pending)
        return tensor

    def locate(self, tensor_id):
        return self._find(tensor_id).meta

    def evict(self, tensor_id, to):
        """Move a tensor to pinned host RAM (the only non-resident tier implemented here)."""
        if to is not MemoryTier.LOCAL_RAM:
            raise NotImplementedError(f"eviction to {to.value} is not implemented")
        if self.locate(tensor_id).tier is MemoryTier.LOCAL_RAM:
            return
        src = self.get(tensor_id)  # also orders after a prefetch still in flight
        staged = torch.empty(src.shape, dtype=src.dtype, pin_memory=torch.cuda.is_available())
        staged.copy_(src)
        with self._mu:
            entry = self._find(tensor_id)
            entry.tensor, entry.meta.tier = staged, MemoryTier.LOCAL_RAM

    def prefetch(self, tensor_id):
        """Start copying an evicted tensor back to its accelerator (async, side stream)."""
        entry = self._find(tensor_id)
        if entry.meta.tier is not MemoryTier.LOCAL_RAM or entry.home.type != "cuda":
            return
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=entry.home)
        with torch.cuda.stream(self._copy_stream):
            back = entry.tensor.to(entry.home, non_blocking=True)
            done = torch.cuda.Event()
            done.record(self._copy_stream)
        with self._mu:
            entry.tensor, entry.ready, entry.meta.tier = back, done, MemoryTier.LOCAL_ACCELERATOR

    def _metas(self) -> list[TensorMeta]:
        with self._mu:
            return [e.meta for e in self._table.values()]

    def ids(self, role: TensorRole | None = None) -> list[str]:
        return sorted(m.tensor_id for m in self._metas() if role in (None, m.role))

    def bytes_by_role(self) -> dict[str, int]:
        totals = dict.fromkeys((r.value for r in TensorRole), 0)
        for m in self._metas():
            totals[m.role.value] += m.bytes
        return totals

    def bytes_by_tier(self) -> dict[str, int]:
        totals: dict[str, int] = {}
        for m in self._metas():
            totals[m.tier.value] = totals.get(m.tier.value, 0) + m.bytes
        return totals

    def manifest(self) -> list[dict]:
        return [m.to_dict() for m in sorted(self._metas(), key=lambda m: m.tensor_id)]

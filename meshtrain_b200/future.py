"""Extension points that are declared but carry no behaviour (reference future.py:1-46).

Tiering (``MemoryTier``), the tensor store and host offload of parameters and
optimizer state are implemented (``parallel/tensor_store.py``,
``parallel/offload.py``), and so is activation recompute: the policies in
``parallel/recompute.py`` implement ``RecomputePolicy``, and link compression:
``networking/compression.py:Downcast`` implements ``CompressionPolicy``, and live
layer migration: ``parallel/migration.py:RebalanceByMeasurement`` implements
``MigrationPolicy``; and the tier of a stage's optimizer state:
``parallel/placement.py:StateTierPolicy`` implements ``PlacementPolicy``.  The
abstract interfaces stay here, where the reference declares them.
"""

from __future__ import annotations

import abc

from meshtrain_b200.parallel.tensor_store import LocalTensorStore, MemoryTier, TensorRole, TensorStore  # noqa: F401


class PlacementPolicy(abc.ABC):
    """Chooses the tier of each tensor from memory pressure and link costs."""

    @abc.abstractmethod
    def place(self, tensor_id: str, nbytes: int, access_pattern: str) -> MemoryTier: ...


class RecomputePolicy(abc.ABC):
    """Which activations to drop in forward and recompute in backward."""

    @abc.abstractmethod
    def should_recompute(self, layer_index: int, saved_bytes: int) -> bool: ...


class CompressionPolicy(abc.ABC):
    """Lossy or lossless encoding of boundary tensors on one link."""

    @abc.abstractmethod
    def encode(self, tensor, link: tuple[str, str]) -> tuple[bytes, dict]: ...

    @abc.abstractmethod
    def decode(self, payload: bytes, meta: dict): ...


class MigrationPolicy(abc.ABC):
    """Moves layers between workers between steps (placements are static today)."""

    @abc.abstractmethod
    def propose(self, step: int, metrics: dict) -> list[tuple[int, str, str]]: ...

"""Where a device-engine stage keeps its fp32 master weights and Adam moments.

The reference declares ``PlacementPolicy.place(key, nbytes, access_pattern) -> MemoryTier``
(future.py:18-23) and keeps every tensor on its accelerator.  Here the optimizer's state of a
stage (fp32 master weights, both Adam moments: 12 bytes per parameter, touched once per
step) is the tensor class that can leave the GPU: ``offload`` settings ``device`` / ``host``
fix the tier, and ``auto`` asks the startup memory estimate whether the stage fits with its
state resident and moves the state to pinned host memory only if it does not.  Weights in
the compute dtype, gradients and activations (touched by every microbatch) stay on the GPU.
"""

from __future__ import annotations

from typing import Callable

from meshtrain_b200.future import PlacementPolicy
from meshtrain_b200.parallel.tensor_store import MemoryTier

MODES = ("device", "host", "auto")


class StateTierPolicy(PlacementPolicy):
    def __init__(self, offload_state: bool):
        self.offload_state = offload_state

    def place(self, tensor_id: str, nbytes: int, access_pattern: str) -> MemoryTier:
        """``access_pattern`` "per_step" (optimizer state) may go to host RAM; anything read
        by every microbatch ("per_microbatch") stays on the accelerator."""
        optimizer_state = access_pattern == "per_step" or ".optim." in tensor_id or tensor_id.endswith(".master")
        if self.offload_state and optimizer_state:
            return MemoryTier.LOCAL_RAM
        return MemoryTier.LOCAL_ACCELERATOR


def decide(mode: str, fits_resident: Callable[[], bool]) -> StateTierPolicy:
    """The policy for an ``offload`` mode; ``fits_resident`` is only asked under "auto"."""
    if mode not in MODES:
        raise ValueError(f"unknown offload mode {mode!r} ({', '.join(MODES)})")
    if mode == "auto":
        return StateTierPolicy(offload_state=not fits_resident())
    return StateTierPolicy(offload_state=mode == "host")


def config_mode(offload_cfg) -> str:
    """One mode from the config's ``offload.params`` / ``offload.optimizer`` (host wins, then auto)."""
    modes = {offload_cfg.params, offload_cfg.optimizer}
    return "host" if "host" in modes else ("auto" if "auto" in modes else "device")

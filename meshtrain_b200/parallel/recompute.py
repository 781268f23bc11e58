"""Activation recompute for the device engine.

A recomputed layer keeps only its input after its forward; its backward first
runs the forward again to re-materialise what the backward reads (normalised
inputs, attention output and log-sum-exp, MLP pre-activations), then frees it.
That trades one extra forward of the layer for its saved activations, which
for a 1F1B stage are held once per microbatch in flight: the lever when a
long-sequence or deep stage does not fit in the GPU's memory.

The reference declares this extension point and leaves it empty
(future.py:26-31, ``RecomputePolicy.should_recompute(layer_index, saved_bytes)``);
the policies here implement that interface.  The embedding (first unit) and
the fused LM head / loss (last unit, whose backward runs inside its forward)
are never recomputed.

Policies by name (``training.activation_recompute``, ``bench.py --recompute``):

    none          keep every activation (default)
    all           recompute every block unit
    every:K       recompute every K-th block unit (global unit index)
    largest:N     recompute the N units with the largest saved activations
"""

from __future__ import annotations

import dataclasses

from meshtrain_b200.future import RecomputePolicy


class KeepActivations(RecomputePolicy):
    def should_recompute(self, layer_index: int, saved_bytes: int) -> bool:
        return False


class RecomputeAll(RecomputePolicy):
    def should_recompute(self, layer_index: int, saved_bytes: int) -> bool:
        return True


class RecomputeEvery(RecomputePolicy):
    def __init__(self, k: int):
        if k < 1:
            raise ValueError("every:K needs K >= 1")
        self.k = k

    def should_recompute(self, layer_index: int, saved_bytes: int) -> bool:
        return layer_index % self.k == 0


class RecomputeLargest(RecomputePolicy):
    """The ``count`` units with the largest saved activations (ties: the earlier unit)."""

    def __init__(self, count: int, saved_by_unit: dict[int, int] | None = None):
        if count < 0:
            raise ValueError("largest:N needs N >= 0")
        self.count = count
        self.chosen: set[int] | None = None
        if saved_by_unit is not None:
            self.rank(saved_by_unit)

    def rank(self, saved_by_unit: dict[int, int]) -> None:
        order = sorted(saved_by_unit, key=lambda u: (-saved_by_unit[u], u))
        self.chosen = set(order[:self.count])

    def should_recompute(self, layer_index: int, saved_bytes: int) -> bool:
        if self.chosen is None:
            raise RuntimeError("RecomputeLargest needs the saved bytes of every unit first (rank())")
        return layer_index in self.chosen


def parse_policy(text: str | None) -> RecomputePolicy:
    """A policy from its name (see the module docstring)."""
    name = (text or "none").strip().lower()
    if name in ("none", "off", "false", "0"):
        return KeepActivations()
    if name in ("all", "full", "true"):
        return RecomputeAll()
    kind, _, arg = name.partition(":")
    if kind == "every" and arg.isdigit():
        return RecomputeEvery(int(arg))
    if kind == "largest" and arg.isdigit():
        return RecomputeLargest(int(arg))
    raise ValueError(f"unknown activation recompute policy {text!r} (none, all, every:K, largest:N)")


def recomputable(num_units: int) -> range:
    """Units that may be recomputed: every one but the embedding and the LM head."""
    return range(1, num_units - 1)


def choose_units(policy: RecomputePolicy | str | None, profiles) -> set[int]:
    """Global units to recompute, from the model's layer profiles (saved bytes per unit)."""
    if not isinstance(policy, RecomputePolicy):
        policy = parse_policy(policy)
    candidates = recomputable(len(profiles))
    if isinstance(policy, RecomputeLargest) and policy.chosen is None:
        policy.rank({u: profiles[u].saved_bytes for u in candidates})
    return {u for u in candidates if policy.should_recompute(u, profiles[u].saved_bytes)}


def apply_to_profiles(profiles, units: set[int]):
    """Profiles as the planner should see them with ``units`` recomputed: such a unit keeps
    only its input across the step, re-materialises its saved bytes during its own backward
    (a transient the estimator counts once), and runs its forward twice."""
    out = []
    for prof in profiles:
        if prof.index in units:
            prof = dataclasses.replace(prof, saved_bytes=prof.input_bytes, recompute_bytes=prof.saved_bytes,
                                       flops=prof.flops * 4.0 / 3.0)  # forward + backward (2x) + forward again
        out.append(prof)
    return out

"""Live layer migration: move stage boundaries between steps from measured stage times.

The reference declares ``MigrationPolicy.propose(step, metrics)`` -> ``[(layer,
from_worker, to_worker)]`` (future.py:46-50) and keeps placements static.  The planner
splits a model by predicted costs (FLOPs, with a fixed weight for attention); when
a stage measures slower or faster than predicted, ``RebalanceByMeasurement``
rescales the predicted cost of every unit by its stage's measured / predicted
ratio, splits again, and proposes the units whose stage changes, if the new split's
largest stage is predicted shorter by more than ``min_gain``.  ``PipelineTrainer.rebalance``
gathers the measurements and carries out a proposal (``repartition``).
"""

from __future__ import annotations

from meshtrain_b200.future import MigrationPolicy


def owner_of(ranges: list[tuple[int, int]]) -> dict[int, int]:
    """Unit -> rank for a plain (one range per rank) layout."""
    return {u: rank for rank, (a, b) in enumerate(ranges) for u in range(a, b)}


class RebalanceByMeasurement(MigrationPolicy):
    def __init__(self, min_gain: float = 0.03):
        self.min_gain = min_gain
        self.last_ranges: list[tuple[int, int]] | None = None
        self.predicted_gain = 0.0

    def new_ranges(self, metrics: dict) -> list[tuple[int, int]] | None:
        """The better split, or None.  ``metrics``: ``ranges`` (current, one per rank),
        ``busy_ms`` (measured work per rank and step) and ``unit_costs`` (predicted)."""
        from meshtrain_b200.parallel.engine import balanced_split

        ranges = [tuple(r) for r in metrics["ranges"]]
        busy, costs = list(metrics["busy_ms"]), list(metrics["unit_costs"])
        if len(busy) != len(ranges) or min(busy) <= 0:
            return None
        corrected = list(costs)
        for (a, b), measured in zip(ranges, busy):
            predicted = sum(costs[a:b]) or 1.0
            for u in range(a, b):
                corrected[u] = costs[u] * measured / predicted
        proposal = balanced_split(corrected, len(ranges))
        now = max(sum(corrected[a:b]) for a, b in ranges)
        then = max(sum(corrected[a:b]) for a, b in proposal)
        self.predicted_gain = (now - then) / now if now > 0 else 0.0
        if proposal == ranges or self.predicted_gain < self.min_gain:
            return None
        self.last_ranges = proposal
        return proposal

    def propose(self, step: int, metrics: dict) -> list[tuple[int, str, str]]:
        proposal = self.new_ranges(metrics)
        if proposal is None:
            return []
        before, after = owner_of(metrics["ranges"]), owner_of(proposal)
        return [(u, f"rank{before[u]}", f"rank{after[u]}") for u in sorted(before) if before[u] != after[u]]

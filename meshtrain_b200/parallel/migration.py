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


def owner_of(ranges: list[tuple[int, int]], ranks: int | None = None) -> dict[int, int]:
    """Unit -> rank; ``ranges`` are the pieces in model order, piece k on rank k mod ``ranks``
    (one piece per rank when ``ranks`` is None)."""
    ranks = ranks or len(ranges)
    return {u: k % ranks for k, (a, b) in enumerate(ranges) for u in range(a, b)}


class RebalanceByMeasurement(MigrationPolicy):
    def __init__(self, min_gain: float = 0.03):
        self.min_gain = min_gain
        self.last_ranges: list[tuple[int, int]] | None = None
        self.predicted_gain = 0.0

    def new_ranges(self, metrics: dict) -> list[tuple[int, int]] | None:
        """The better split, or None.  ``metrics``: ``ranges`` (the pieces in model order; piece k on
        rank k mod the number of ranks), ``busy_ms`` (measured work per rank and step), ``unit_costs``
        (predicted) and, for interleaved layouts, ``chunks`` (pieces per rank)."""
        from meshtrain_b200.parallel.engine import balanced_split, interleaved_split

        ranges = [tuple(r) for r in metrics["ranges"]]
        busy, costs = list(metrics["busy_ms"]), list(metrics["unit_costs"])
        chunks = int(metrics.get("chunks", 1))
        ranks = len(busy)
        if ranks * chunks != len(ranges) or min(busy) <= 0:
            return None
        owner = owner_of(ranges, ranks)
        predicted = [0.0] * ranks
        for u, rank in owner.items():
            predicted[rank] += costs[u]
        # every unit of a rank is scaled by that rank's measured / predicted work
        corrected = [costs[u] * busy[owner[u]] / (predicted[owner[u]] or 1.0) for u in range(len(costs))]

        def worst(pieces):
            per_rank = [0.0] * ranks
            for k, (a, b) in enumerate(pieces):
                per_rank[k % ranks] += sum(corrected[a:b])
            return max(per_rank)

        proposal = balanced_split(corrected, ranks) if chunks == 1 else interleaved_split(corrected, ranks, chunks)
        now, then = worst(ranges), worst(proposal)
        self.predicted_gain = (now - then) / now if now > 0 else 0.0
        if proposal == ranges or self.predicted_gain < self.min_gain:
            return None
        self.last_ranges = proposal
        return proposal

    def propose(self, step: int, metrics: dict) -> list[tuple[int, str, str]]:
        proposal = self.new_ranges(metrics)
        if proposal is None:
            return []
        ranks = len(metrics["busy_ms"])
        before, after = owner_of(metrics["ranges"], ranks), owner_of(proposal, ranks)
        return [(u, f"rank{before[u]}", f"rank{after[u]}") for u in sorted(before) if before[u] != after[u]]

"""Partition planning: layer profiles, cost model, memory estimator, placement."""

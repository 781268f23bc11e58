"""Experiments: correctness oracles, placement studies, capacity sweeps, device checks."""

"""Hardware detection, device micro-benchmarks and link probes."""

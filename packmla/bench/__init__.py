"""Benchmarks: device timing helpers, clock sampling, synthetic serving state, microbenchmarks."""

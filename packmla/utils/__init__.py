"""Utilities: metrics, NVTX ranges, run records."""

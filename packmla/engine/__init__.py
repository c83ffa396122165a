"""Serving engine: request state, scheduler, CUDA-graph decode runner, sampler."""

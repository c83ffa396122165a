"""Parallelism: process groups, NCCL baseline collectives, symmetric memory, fused kernels."""

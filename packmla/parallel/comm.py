"""Tensor/expert-parallel communicator.

The NCCL all-reduce is the baseline (reference: SGLang TP groups over NCCL, Dockerfile.v0.5.22:79-84).
The fused GEMM + all-reduce kernels over NVLink peer memory live in packmla/parallel/fused.py and
replace these calls when enabled.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0):
    """Initialise torch.distributed from RANK/WORLD_SIZE/MASTER_* (torchrun); returns (rank, world, local_rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


class TPComm:
    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        """[rows, ...] from every rank -> [world * rows, ...] in rank order (equal rows on every rank)."""
        if self.world == 1:
            return t
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:
            dist.all_gather(list(out.chunk(self.world)), t.contiguous(), group=self.group)
        return out

    def reduce_scatter_rows(self, t: torch.Tensor) -> torch.Tensor:
        """[world * rows, ...] partial sums from every rank -> this rank's [rows, ...] block of the sum."""
        if self.world == 1:
            return t
        rows = t.shape[0] // self.world
        if dist.get_backend(self.group) == "nccl":
            out = torch.empty((rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            dist.reduce_scatter_tensor(out, t.contiguous(), group=self.group)
            return out
        full = t.contiguous().clone()
        dist.all_reduce(full, group=self.group)
        return full[self.rank * rows:(self.rank + 1) * rows].contiguous()

    def exchange_ints(self, vals: list[int], device) -> list[list[int]]:
        """Every rank's small list of ints (same length on every rank), in rank order."""
        if self.world == 1:
            return [list(vals)]
        dev = device if dist.get_backend(self.group) == "nccl" else "cpu"
        t = torch.tensor(vals, dtype=torch.int64, device=dev)
        out = torch.empty(self.world * len(vals), dtype=torch.int64, device=dev)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(out, t, group=self.group)
        else:
            dist.all_gather(list(out.chunk(self.world)), t, group=self.group)
        flat = out.tolist()
        return [flat[i * len(vals):(i + 1) * len(vals)] for i in range(self.world)]

    def max_over_ranks(self, v: float, device) -> float:
        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def sum_over_ranks(self, v: float, device) -> float:
        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, group=self.group)
        return float(t.item())

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

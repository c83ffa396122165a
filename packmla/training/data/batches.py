"""Device staging of training states, one batch at a time, plus the frozen codec-anchor bank.

Sources stay caller-owned CPU tensors (normally memory-mapped cache pages); only the current batch
lives on the device (reference: training/data/batches.py `StateBatches`).  Anchors (codec residuals
of the warm scorer, anchored recipe only) are computed once, in training order, and kept in a
temporary file-backed fp32 bank so they never occupy device memory between batches.
"""
from __future__ import annotations

import tempfile
from contextlib import contextmanager
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Sequence

import torch


@dataclass
class StagedBatch:
    states: list[dict]
    anchors: list[dict] | None = None


def _to(state: dict, device: torch.device) -> dict:
    return {k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) and k != "target_unrounded" else v)
            for k, v in state.items() if k != "target_unrounded"}


class StateBatches:
    def __init__(self, states: Sequence[dict], device, limit: int, scratch_root: Path | None = None):
        if not states or limit < 1:
            raise ValueError("nonempty states and positive staging limit required")
        self.states = states
        self.device = torch.device(device)
        self.limit = limit
        self.scratch_root = scratch_root
        self.anchor_bytes = 0
        self._bank: dict | None = None
        self._tmp = None

    def __enter__(self) -> "StateBatches":
        return self

    def __exit__(self, *exc) -> None:
        self._bank = None
        if self._tmp is not None:
            self._tmp.cleanup()
            self._tmp = None

    def prepare_anchors(self, make: Callable[[dict], dict]) -> None:
        """Compute one anchor per state (on the device, one state at a time) into a mapped bank."""
        self._tmp = tempfile.TemporaryDirectory(prefix="anchors-", dir=self.scratch_root)
        rows, outs = [], []
        for s in self.states:
            st = _to({**s}, self.device)
            a = make(st)
            rows.append(a["rows"].float().cpu())
            outs.append(a["output"].float().cpu())
        path = Path(self._tmp.name) / "anchors.pt"
        torch.save({"rows": rows, "output": outs}, path)
        self._bank = torch.load(path, mmap=True, weights_only=True)
        self.anchor_bytes = sum(t.numel() * 4 for t in rows + outs)

    @contextmanager
    def stage(self, indices, with_anchors: bool = True):
        idx = [int(i) for i in indices]
        if not idx or len(idx) > self.limit:
            raise ValueError("batch larger than the staging limit")
        states = [_to(self.states[i], self.device) for i in idx]
        anchors = None
        if with_anchors and self._bank is not None:
            anchors = [{"state": st, "rows": self._bank["rows"][i].to(self.device),
                        "output": self._bank["output"][i].to(self.device)} for st, i in zip(states, idx)]
        try:
            yield StagedBatch(states, anchors)
        finally:
            del states, anchors

"""Loader of the in-tree CUDA extension `packmla._C`.

CUDA tensors always go through the extension; if it is missing the call fails
loudly (no silent PyTorch fallback).  CPU tensors use the fp32 oracle instead.
"""
from __future__ import annotations

import torch

_EXT = None
_ERR: dict[int, torch.Tensor] = {}


# split counts whose decode CTAs form one thread-block cluster and merge in distributed shared memory
# (one launch); other counts above one write partials that a second (combine) kernel merges
CLUSTER_SPLITS = (2, 4, 8)


def decode_uses_partials(splits: int) -> bool:
    return splits > 1 and splits not in CLUSTER_SPLITS


# kernels launched per extension entry point (for the bench's launch count): a number, or a function of
# the call's positional arguments
KERNELS_PER_CALL = {"native_store": 1, "packed_store": 1,
                    "sparse_mla_decode": lambda a: 2 if decode_uses_partials(int(a[16])) else 1, "moe_fp4": 3, "moe_fp4_mma": 4, "add_rmsnorm": 1, "bs_probe": 1, "moe_mxf4": 4, "bs_probe2": 1, "rope_q": 1, "comp_pool": 1, "route_topk": 1, "silu_mul": 1, "index_key_store": 1, "index_select": 2, "umma_probe": 1, "gemm_allreduce": 1, "allreduce": 1}


class _Counting:
    """Proxy that counts kernel launches of extension calls while `enabled`."""

    def __init__(self, mod):
        self._mod = mod
        self.enabled = False
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not self.enabled:
            return fn
        per = KERNELS_PER_CALL.get(name, 1)

        def wrapped(*a, **k):
            self.launches += per(a) if callable(per) else per
            return fn(*a, **k)

        return wrapped


def ext():
    global _EXT
    if _EXT is None:
        try:
            from packmla import _C  # noqa: WPS433
        except ImportError as exc:  # pragma: no cover - exercised on GPU boxes only
            raise RuntimeError(
                "packmla CUDA extension is not built; run `python setup.py build_ext --inplace`"
            ) from exc
        import os
        import warnings

        from ..utils.source_digest import check_record

        stale = check_record(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        if stale:
            warnings.warn(stale, RuntimeWarning, stacklevel=2)
        _EXT = _Counting(_C)
    return _EXT


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32[4] error word written by kernels instead of trapping."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = t
    return t


ERROR_NAMES = {1: "bounded wait timed out", 2: "index out of range", 3: "bad argument", 4: "peer timed out"}


def check_errors(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronize and raise if any kernel on `device` reported an error."""
    devs = [device] if device is not None else [torch.device("cuda", i) for i in list(_ERR)]
    for d in devs:
        w = error_word(d)
        vals = w.tolist()
        if reset:
            w.zero_()
        if vals[0] != 0:
            raise RuntimeError(
                f"packmla kernel error on {d}: {ERROR_NAMES.get(vals[0], vals[0])} "
                f"(block {vals[1]}, detail {vals[2]}, count {vals[3]})"
            )

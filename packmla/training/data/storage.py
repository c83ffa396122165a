"""Storage audit of a training cache: byte accounting per layer and tensor kind, and read timing.

    python -m packmla.training.data.storage --cache CACHE [--repeat 3]

Reference: training/data/storage.py (`audit` byte accounting of capture payloads, reader benchmarks).
For each cached layer: file bytes, tensor bytes by kind (raw C4 rows, RoPE tables, queries, SWA rows,
targets, ...) summed over its states, the state count per role, and the time to open the layer through
the checksum-verified, memory-mapped reader (`load_cached_layer`) and to touch every tensor once.
"""
from __future__ import annotations

import argparse
import json
import time
from collections import defaultdict
from pathlib import Path

import torch

from .cache import layer_file, load_cached_layer


def _tensor_bytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def audit(cache: Path, repeat: int = 1) -> dict:
    cache = Path(cache)
    config = json.loads((cache / "config.json").read_text())
    layers = {}
    totals: dict[str, int] = defaultdict(int)
    for layer in config["layers"]:
        open_s, touch_s = [], []
        for _ in range(max(1, repeat)):
            t0 = time.perf_counter()
            roles = load_cached_layer(cache, layer)
            t1 = time.perf_counter()
            kinds: dict[str, int] = defaultdict(int)
            checksum = 0.0
            for rows in roles.values():
                for s in rows:
                    for k, v in s.items():
                        if isinstance(v, torch.Tensor):
                            kinds[k] += _tensor_bytes(v)
                            checksum += float(v.abs().sum())  # touches every element of the mapped pages
            touch_s.append(time.perf_counter() - t1)
            open_s.append(t1 - t0)
        file_bytes = (cache / layer_file(layer)).stat().st_size
        tensor_bytes = sum(kinds.values())
        for k, v in kinds.items():
            totals[k] += v
        layers[str(layer)] = {"file_bytes": file_bytes, "tensor_bytes": tensor_bytes,
                              "overhead_bytes": file_bytes - tensor_bytes, "by_kind": dict(sorted(kinds.items())),
                              "states": {r: len(v) for r, v in roles.items()},
                              "open_verify_s": min(open_s), "touch_s": min(touch_s),
                              "touch_GBps": tensor_bytes / max(min(touch_s), 1e-9) / 1e9}
    return {"cache": str(cache.resolve()), "layers": layers, "total_by_kind": dict(sorted(totals.items())),
            "total_tensor_bytes": sum(totals.values()),
            "total_file_bytes": sum(v["file_bytes"] for v in layers.values())}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--cache", type=Path, required=True)
    ap.add_argument("--repeat", type=int, default=3)
    a = ap.parse_args(argv)
    out = audit(a.cache, a.repeat)
    print(json.dumps(out, indent=2))
    return out


if __name__ == "__main__":
    main()

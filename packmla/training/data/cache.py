"""Hash-bound training cache of captured decode queries (one file per C4 layer).

Layout of a cache directory (reference: repo-root data/training-cache-001, training/data/dataset.py
`load_layer` / `load_cached_layer` / `validate_states`):

    config.json    {"format": "packmla-training-cache", "version": 1, "layers": [...],
                    "split": {"train": [rids], "development": [rids], "test": []},
                    "queries": {"train": n, "development": m}, "model": {...}}
    index.json     {"layer-XX.pt": sha256 of the file}
    progress.json  {"status": "complete", "layers": [...]}
    layer-XX.pt    torch.save({"train": [state], "development": [state]})  (default zip format, so it
                   memory-maps)

A state is one captured decode query of one layer:
    rid, ordinal, split, role                         identity
    raw [R,512] f32, freq [R,32] c64                  selected C4 records' compressor rows and RoPE
    weight [512] f32, eps                             the layer's KV RMSNorm
    q [H,512] f32, sink [H] f32, scale                the query (tail rotated) and softmax constants
    swa [W,512] f32                                   decoded Native SWA rows (rotated)
    query_freq [32] c64                               RoPE of the query position
    target [H,512] f32, reference_squared_norm        Native-record attention output (BF16, inverse
                                                      RoPE) and its squared norm
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from ..calibration import Math, file_sha256

FORMAT = "packmla-training-cache"
FLOAT_KEYS = ("raw", "weight", "q", "swa", "sink", "target")
COMPLEX_KEYS = ("freq", "query_freq")


def layer_file(layer: int) -> str:
    return f"layer-{layer:02d}.pt"


def validate_state(s: dict) -> None:
    R = s["raw"].shape[0]
    H = s["q"].shape[0]
    shapes = {"raw": (R, 512), "freq": (R, 32), "weight": (512,), "q": (H, 512), "sink": (H,),
              "target": (H, 512), "query_freq": (32,)}
    for k, shp in shapes.items():
        t = s[k]
        if not isinstance(t, torch.Tensor) or tuple(t.shape) != shp or not bool(torch.isfinite(
                torch.view_as_real(t) if t.is_complex() else t).all()):
            raise ValueError(f"{s.get('rid')}/{s.get('ordinal')}: bad or nonfinite {k}")
    if s["swa"].dim() != 2 or s["swa"].shape[1] != 512:
        raise ValueError("swa rows must be [W, 512]")
    for k in FLOAT_KEYS:
        if s[k].dtype != torch.float32:
            raise ValueError(f"{k} must be float32")
    for k in COMPLEX_KEYS:
        if s[k].dtype != torch.complex64:
            raise ValueError(f"{k} must be complex64")
    den = s["reference_squared_norm"]
    if not np.isfinite(den) or den <= 0 or abs(den - float(s["target"].double().square().sum())) > 1e-5 * den:
        raise ValueError("native target denominator changed")
    if not (np.isfinite(s["eps"]) and s["eps"] > 0 and np.isfinite(s["scale"]) and s["scale"] > 0):
        raise ValueError("positive normalization/attention constants required")


def write_cache(root: Path, states_by_layer: dict[int, dict[str, list[dict]]], split: dict, queries: dict,
                model: dict | None = None) -> None:
    """Write a complete cache (refuses an existing directory: caches are immutable)."""
    root = Path(root)
    if root.exists():
        raise ValueError(f"fresh cache directory required: {root}")
    root.mkdir(parents=True)
    index = {}
    for layer, roles in sorted(states_by_layer.items()):
        for role, rows in roles.items():
            for s in rows:
                validate_state(s)
                if s["role"] != role:
                    raise ValueError("state role mismatch")
        path = root / layer_file(layer)
        torch.save(roles, path)
        index[path.name] = file_sha256(path)
    Math.atomic_json(root / "config.json", {"format": FORMAT, "version": 1, "layers": sorted(states_by_layer),
                                            "split": split, "queries": queries, "model": model or {}})
    Math.atomic_json(root / "index.json", index)
    Math.atomic_json(root / "progress.json", {"status": "complete", "layers": sorted(states_by_layer)})


def load_cached_layer(root: Path, layer: int) -> dict[str, list[dict]]:
    """Checksum-verified, memory-mapped states of one layer, validated against the frozen split."""
    root = Path(root)
    config = json.loads((root / "config.json").read_text())
    progress = json.loads((root / "progress.json").read_text())
    if config.get("format") != FORMAT or progress.get("status") != "complete":
        raise ValueError(f"complete packmla training cache required: {root}")
    if layer not in config["layers"]:
        raise ValueError(f"layer {layer} not in cache")
    path = root / layer_file(layer)
    expected = json.loads((root / "index.json").read_text()).get(path.name)
    if expected is None or file_sha256(path) != expected:
        raise ValueError(f"cache payload changed: {path}")
    roles = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
    if set(roles) != {"train", "development"}:
        raise ValueError("explicit train/development roles required")
    split = config["split"]
    if set(split["train"]) & set(split["development"]) or split.get("test"):
        raise ValueError("disjoint development split and no fresh-test claim required")
    for role, rows in roles.items():
        keys = [(s["rid"], s["ordinal"]) for s in rows]
        if len(set(keys)) != len(keys) or {r for r, _ in keys} != set(split[role]):
            raise ValueError(f"{role}: frozen issue coverage changed")
        per = config["queries"][role]
        if any(sum(r == rid for r, _ in keys) != per for rid in split[role]):
            raise ValueError(f"{role}: {per} queries per issue required")
        for s in rows:
            if s["role"] != role:
                raise ValueError("state role mismatch")
            validate_state(s)
    return roles


def frozen_split(ids: list[str], development: int, seed: int = 42) -> dict:
    """Deterministic issue split: `development` issues for selection, the rest for fitting."""
    order = list(np.random.default_rng(seed).permutation(sorted(ids)))
    return {"train": sorted(order[development:]), "development": sorted(order[:development]), "test": []}

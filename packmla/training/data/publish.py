"""Published raw captures: per-issue bundles bound to one capture configuration, a verifying reader with
bounded reads, cache building from publications, and coverage extension of an existing cache.

Reference behaviour (training/data/dataset.py): captured states are published per issue (a marker naming a
bundle, a receipt holding the capture configuration's sha256); the reader verifies every requested issue's
publication before use and again when it reads, keeps at most one rank group of bytes (256 MiB) in memory and
checks them against their hashes; `extend_coverage` adds training queries to a complete cache from the same
hash-bound captures while every original state stays byte-identical.  The layout here is packmla's own:

    capture-config.json                  the capture configuration (model, layers, split, queries captured)
    bundles/<rid>/layer-XX.pt            torch.save([state, ...]) of one issue and layer, every captured query
    published/<rid>.json                 {"bundle": "bundles/<rid>", "files": {"layer-XX.pt": sha256},
                                          "receipt": {"capture_config_sha256": ...}}

A marker is written last and atomically, so an issue is published or not; files are never rewritten.
"""
from __future__ import annotations

import hashlib
import io
import json
import os
from dataclasses import dataclass
from pathlib import Path

import torch

from ..calibration import Math, file_sha256
from .cache import layer_file, load_cached_layer, validate_state, write_cache

MAX_GROUP_BYTES = 256 * 1024 ** 2  # bytes of one issue-layer bundle held at once


def _signature(path: Path) -> tuple[int, ...]:
    """Identity and state of a file (access time left out: reading must not change it)."""
    st = path.stat()
    return st.st_dev, st.st_ino, st.st_size, st.st_mtime_ns, st.st_ctime_ns


def _atomic_bytes(path: Path, data: bytes) -> None:
    tmp = path.with_name(path.name + f".tmp-{os.getpid()}")
    with open(tmp, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def write_capture_config(root: Path, config: dict) -> str:
    """Create a publication root with its capture configuration; returns the configuration's sha256."""
    root = Path(root)
    if (root / "capture-config.json").exists():
        raise ValueError(f"publication root already configured: {root}")
    (root / "bundles").mkdir(parents=True, exist_ok=True)
    (root / "published").mkdir(exist_ok=True)
    Math.atomic_json(root / "capture-config.json", config)
    return file_sha256(root / "capture-config.json")


def publish_issue(root: Path, rid: str, states_by_layer: dict[int, list[dict]]) -> dict:
    """Publish one issue's captured states (every layer of the capture); refuses a republication."""
    root = Path(root)
    config = json.loads((root / "capture-config.json").read_text())
    if rid not in config["requests"]:
        raise ValueError(f"issue absent from the capture configuration: {rid}")
    marker = root / "published" / f"{rid}.json"
    bundle = root / "bundles" / rid
    if marker.exists() or bundle.exists():
        raise ValueError(f"issue already published: {rid}")
    if set(states_by_layer) != set(config["layers"]):
        raise ValueError("every captured layer of the configuration required")
    bundle.mkdir(parents=True)
    files = {}
    for layer, states in sorted(states_by_layer.items()):
        for s in states:
            if s["rid"] != rid:
                raise ValueError("state of another issue in the bundle")
            validate_state(s)
        buf = io.BytesIO()
        torch.save(states, buf)
        data = buf.getvalue()
        if len(data) > MAX_GROUP_BYTES:
            raise ValueError(f"bundle of layer {layer} exceeds {MAX_GROUP_BYTES} bytes")
        _atomic_bytes(bundle / layer_file(layer), data)
        files[layer_file(layer)] = hashlib.sha256(data).hexdigest()
    record = {"bundle": f"bundles/{rid}", "files": files,
              "receipt": {"capture_config_sha256": file_sha256(root / "capture-config.json"), "issue": rid}}
    _atomic_bytes(marker, json.dumps(record, indent=1, sort_keys=True).encode())
    return record


@dataclass(frozen=True)
class _Proof:
    record: dict
    marker_bytes: bytes
    signatures: dict[str, tuple[int, ...]]


class PublishedCaptures:
    """Verified view of some issues' publications.  Every requested issue must be published under the
    root's capture configuration; a bundle file is read (bounded, hash-checked) only while its marker, its
    signature and the configuration are the ones verified.  One reader per caller (not thread-safe)."""

    def __init__(self, root: Path, issues: list[str], max_bytes: int = MAX_GROUP_BYTES):
        if not issues or len(set(issues)) != len(issues):
            raise ValueError("nonempty unique issues required")
        self.root = Path(root).resolve()
        self.max_bytes = max_bytes
        self.config_bytes = (self.root / "capture-config.json").read_bytes()
        self.config = json.loads(self.config_bytes)
        cfg_sha = hashlib.sha256(self.config_bytes).hexdigest()
        self._proof: dict[str, _Proof] = {}
        missing = []
        for rid in issues:
            if rid not in self.config["requests"]:
                raise ValueError(f"issue absent from the capture configuration: {rid}")
            marker = self.root / "published" / f"{rid}.json"
            if not marker.exists():
                missing.append(rid)
                continue
            try:
                marker_bytes = marker.read_bytes()
                record = json.loads(marker_bytes)
                bundle = (self.root / record["bundle"]).resolve()
                if not bundle.is_relative_to(self.root):
                    raise ValueError("bundle outside the publication root")
                if record["receipt"]["capture_config_sha256"] != cfg_sha:
                    raise ValueError("published under another capture configuration")
                if set(record["files"]) != {layer_file(layer) for layer in self.config["layers"]}:
                    raise ValueError("bundle does not cover the configured layers")
                sigs = {}
                for name, sha in record["files"].items():
                    path = bundle / name
                    before = _signature(path)
                    if file_sha256(path) != sha or _signature(path) != before:
                        raise ValueError(f"bundle file changed or differs from its hash: {name}")
                    sigs[name] = before
                if marker.read_bytes() != marker_bytes:
                    raise ValueError("marker changed during verification")
                self._proof[rid] = _Proof(record, marker_bytes, sigs)
            except (OSError, KeyError, ValueError) as e:
                raise ValueError(f"invalid publication of {rid}: {e}") from e
        if missing:
            raise ValueError(f"unpublished issues: {', '.join(missing)}")

    def _check(self, rid: str) -> _Proof:
        proof = self._proof.get(rid)
        if proof is None:
            raise ValueError(f"issue outside the verified coverage: {rid}")
        if ((self.root / "published" / f"{rid}.json").read_bytes() != proof.marker_bytes
                or (self.root / "capture-config.json").read_bytes() != self.config_bytes):
            raise ValueError(f"publication of {rid} changed after verification")
        return proof

    def load(self, rid: str, layer: int) -> list[dict]:
        """The issue's captured states of one layer (validated; identity checked)."""
        proof = self._check(rid)
        name = layer_file(layer)
        if name not in proof.record["files"]:
            raise ValueError(f"layer {layer} not captured")
        path = (self.root / proof.record["bundle"]).resolve() / name
        if _signature(path) != proof.signatures[name]:
            raise ValueError(f"bundle file changed after verification: {rid}/{name}")
        with open(path, "rb") as f:
            data = f.read(self.max_bytes + 1)
        if len(data) > self.max_bytes:
            raise ValueError(f"bundle file exceeds {self.max_bytes} bytes: {rid}/{name}")
        if hashlib.sha256(data).hexdigest() != proof.record["files"][name]:
            raise ValueError(f"bundle payload changed: {rid}/{name}")
        states = torch.load(io.BytesIO(data), map_location="cpu", weights_only=True)
        del data  # one bundle's bytes at a time
        for s in states:
            if s["rid"] != rid:
                raise ValueError(f"capture identity mismatch in {rid}/{name}")
            validate_state(s)
        self._check(rid)
        return states


def _select(states: list[dict], n: int, rid: str, role: str) -> list[dict]:
    """The first n captured queries of an issue (ordinal order), tagged with the role."""
    rows = sorted(states, key=lambda s: s["ordinal"])
    if len(rows) < n:
        raise ValueError(f"{rid}: {n} {role} queries requested, {len(rows)} captured")
    return [{**s, "role": role, "split": role} for s in rows[:n]]


def build_cache(root: Path, output: Path, queries: dict[str, int]) -> dict:
    """A training cache from the verified publications of the configuration's split."""
    cfg = json.loads((Path(root) / "capture-config.json").read_text())
    split = cfg["split"]
    reader = PublishedCaptures(root, split["train"] + split["development"])
    by_layer = {}
    for layer in cfg["layers"]:
        roles = {"train": [], "development": []}
        for role in ("train", "development"):
            for rid in split[role]:
                roles[role] += _select(reader.load(rid, layer), queries[role], rid, role)
        by_layer[layer] = roles
    write_cache(Path(output), by_layer, split, dict(queries),
                {**cfg.get("model", {}), "capture_config_sha256": file_sha256(Path(root) / "capture-config.json")})
    return {"cache": str(output), "layers": cfg["layers"], "queries": dict(queries)}


def _same_state(a: dict, b: dict) -> bool:
    for k, v in a.items():
        w = b.get(k)
        if isinstance(v, torch.Tensor):
            if not isinstance(w, torch.Tensor) or v.dtype != w.dtype or v.shape != w.shape or not torch.equal(v, w):
                return False
        elif v != w:
            return False
    return set(a) == set(b)


def extend_coverage(root: Path, base_cache: Path, output: Path, train_queries: int,
                    layers: list[int] | None = None) -> dict:
    """A new cache with `train_queries` training queries per issue: the base cache's training and
    development states unchanged (checked tensor by tensor), the added training queries taken only from the
    verified publications of the same capture configuration.  CPU only; no new issues, no new targets."""
    base_cache, output = Path(base_cache), Path(output)
    if output.exists():
        raise ValueError(f"fresh output directory required: {output}")
    base_cfg = json.loads((base_cache / "config.json").read_text())
    cap_sha = base_cfg.get("model", {}).get("capture_config_sha256")
    if cap_sha is None or cap_sha != file_sha256(Path(root) / "capture-config.json"):
        raise ValueError("the base cache was not built from this capture configuration")
    if train_queries <= base_cfg["queries"]["train"]:
        raise ValueError("an extension adds training queries")
    layers = list(layers or base_cfg["layers"])
    if not set(layers) <= set(base_cfg["layers"]):
        raise ValueError("layers outside the base cache")
    split = base_cfg["split"]
    reader = PublishedCaptures(root, split["train"] + split["development"])
    by_layer, added = {}, 0
    for layer in layers:
        base = load_cached_layer(base_cache, layer)
        train = []
        for rid in split["train"]:
            old = [s for s in base["train"] if s["rid"] == rid]
            new = _select(reader.load(rid, layer), train_queries, rid, "train")
            for s_old, s_new in zip(sorted(old, key=lambda s: s["ordinal"]), new):
                if not _same_state(s_old, s_new):
                    raise ValueError(f"original training state changed: {rid}/{s_old['ordinal']} layer {layer}")
            train += new
            added += len(new) - len(old)
        by_layer[layer] = {"train": train, "development": [dict(s) for s in base["development"]]}
    queries = {"train": train_queries, "development": base_cfg["queries"]["development"]}
    write_cache(output, by_layer, split, queries,
                {**base_cfg.get("model", {}), "extended_from": str(base_cache),
                 "base_index_sha256": file_sha256(base_cache / "index.json")})
    return {"cache": str(output), "layers": layers, "queries": queries, "added_states": added}

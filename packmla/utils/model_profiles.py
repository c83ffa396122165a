"""Pinned identities of the model families the reference serves, verified offline against a local checkpoint.

    python -m packmla.utils.model_profiles list
    python -m packmla.utils.model_profiles verify dsv4 /path/to/DeepSeek-V4-Flash-0731

Reference behaviour: scripts/model_profiles.py pins, per family, the Hugging Face repository and revision,
the sha256 of its config.json, the shard count, the checkpoint size and the metadata files a deployment
needs.  The identities are facts about those public repositories, so they are the same here; what packmla
adds is the offline check of a downloaded directory (no network: the config's bytes are hashed, the index's
shards counted and the metadata files required) and the packmla model config a family maps to.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from dataclasses import asdict, dataclass
from pathlib import Path


@dataclass(frozen=True)
class ModelProfile:
    family: str
    repository: str
    revision: str
    config_sha256: str
    shards: int
    checkpoint_bytes: int | None
    metadata_files: tuple[str, ...]
    packmla_config: str | None  # `packmla.server.__main__.model_config` name, where packmla serves the family

    @property
    def config_url(self) -> str:
        return f"https://huggingface.co/{self.repository}/resolve/{self.revision}/config.json"


PROFILES = {
    "dsv4": ModelProfile("dsv4", "deepseek-ai/DeepSeek-V4-Flash-0731", "7872f01b1d1fe23eabc4c98b48bffcef5a386062",
                         "6c8f3d2d3b48707541b88f32f22ef3f0f8a6b57d8523281e2b8d3cdb0ae9a023", 48, None,
                         ("config.json", "model.safetensors.index.json"), "v4-flash"),
    "dsv41": ModelProfile("dsv41", "deepseek-ai/DeepSeek-V4.1-Flash-1017", "1bae0e1088993b9b82de08f59de5be5a34e42170",
                          "8be45ce0476004a3f529fd896115a4a2e800a129ad2d3ec05b16050f52e21879", 48, 510_296_708_312,
                          ("config.json", "model.safetensors.index.json", "tokenizer.json", "tokenizer_config.json"),
                          None),
    "glm53": ModelProfile("glm53", "zai-org/GLM-5.3-Flash", "46a050bec13002ad29ee795c16e61cf4fa3c4a9c",
                          "bb8f01c42cb92a52ca72e65afb4d5bd8d11aef083cd210e8de25dfb904f23e9f", 62, 328_337_455_672,
                          ("config.json", "model.safetensors.index.json", "tokenizer.json", "tokenizer_config.json",
                           "chat_template.jinja"), None),
}


def profile(family: str) -> ModelProfile:
    if family not in PROFILES:
        raise ValueError(f"unknown model family {family!r}; known: {', '.join(sorted(PROFILES))}")
    return PROFILES[family]


def verify_checkpoint(family: str, directory: Path, check_bytes: bool = False) -> dict:
    """Raise ValueError unless `directory` holds the pinned checkpoint: metadata files present, config.json
    bytes with the pinned sha256, the index naming the pinned number of shards (all present), and with
    `check_bytes` the pinned total size of the shards."""
    p = profile(family)
    d = Path(directory)
    missing = [f for f in p.metadata_files if not (d / f).is_file()]
    if missing:
        raise ValueError(f"{family}: missing metadata files {missing} in {d}")
    digest = hashlib.sha256((d / "config.json").read_bytes()).hexdigest()
    if digest != p.config_sha256:
        raise ValueError(f"{family}: config.json sha256 {digest} is not the pinned {p.config_sha256} ({p.revision})")
    index = json.loads((d / "model.safetensors.index.json").read_text())
    shards = sorted(set(index.get("weight_map", {}).values()))
    if len(shards) != p.shards:
        raise ValueError(f"{family}: the index names {len(shards)} shards, pinned {p.shards}")
    absent = [s for s in shards if not (d / s).is_file()]
    if absent:
        raise ValueError(f"{family}: {len(absent)} shards absent, first {absent[0]}")
    total = sum((d / s).stat().st_size for s in shards)
    if check_bytes and p.checkpoint_bytes is not None and total != p.checkpoint_bytes:
        raise ValueError(f"{family}: shards hold {total} bytes, pinned {p.checkpoint_bytes}")
    return {"family": family, "revision": p.revision, "config_sha256": digest, "shards": len(shards),
            "bytes": total}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("list")
    v = sub.add_parser("verify")
    v.add_argument("family")
    v.add_argument("directory", type=Path)
    v.add_argument("--check-bytes", action="store_true")
    a = ap.parse_args(argv)
    if a.cmd == "list":
        print(json.dumps({k: {**asdict(p), "config_url": p.config_url} for k, p in PROFILES.items()}, indent=1))
        return 0
    try:
        print(json.dumps(verify_checkpoint(a.family, a.directory, a.check_bytes)))
        return 0
    except ValueError as e:
        print(f"model profile: {e}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())

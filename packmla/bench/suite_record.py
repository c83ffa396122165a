"""Resumable suite records: JSON-line results bound to the sources, library and fixture they were measured with.

Reference behaviour: the GLM timing suite's `--resume` accepts a partial run only with a verified build
manifest whose source, artifact and fixture identities match the current ones (third_party/README.md:473-476,
scripts/modal/kernels.py:2637-2660).  Here a suite writing to `OUT.jsonl` first writes `OUT.manifest.json`:
the compiled-source digest, the library's hash and the digest it was built from, and the suite's fixture
parameters (seed, shapes, rounds).  A fresh run refuses an existing file.  `resume=True` requires both files.
The manifest must match the current identity field by field.  Cases already recorded are skipped, and new
rows are appended.
"""
from __future__ import annotations

import json
from pathlib import Path

IDENTITY_KEYS = ("csrc_sha256", "library_sha256", "library_built_from")


def current_identity() -> dict:
    from ..utils.provenance import source_identity

    ident = source_identity()
    return {"csrc_sha256": ident["csrc_sha256"], "library_sha256": ident["library"]["sha256"],
            "library_built_from": ident["library"]["built_from_sha256"]}


class SuiteRecord:
    def __init__(self, path, fixture: dict, resume: bool = False, identity: dict | None = None):
        self.path = Path(path)
        self.manifest_path = self.path.with_name(self.path.name + ".manifest.json")
        ident = identity if identity is not None else current_identity()
        manifest = {"identity": {k: ident.get(k) for k in IDENTITY_KEYS}, "fixture": fixture}
        self.done: set[str] = set()
        if resume:
            if not self.path.exists() or not self.manifest_path.exists():
                raise ValueError(f"nothing to resume: {self.path} or its manifest is missing")
            saved = json.loads(self.manifest_path.read_text())
            for part in ("identity", "fixture"):
                for k, v in manifest[part].items():
                    if saved.get(part, {}).get(k) != v:
                        raise ValueError(f"cannot resume: {part} field {k!r} differs ({saved.get(part, {}).get(k)!r} "
                                         f"recorded, {v!r} now)")
                if set(saved.get(part, {})) != set(manifest[part]):
                    raise ValueError(f"cannot resume: the recorded {part} has other fields")
            text = self.path.read_text()
            if text and not text.endswith("\n"):  # an interrupted write: drop the partial line
                text = text[:text.rfind("\n") + 1]
                self.path.write_text(text)
            for line in text.splitlines():
                line = line.strip()
                if line.startswith("{"):
                    try:
                        self.done.add(json.loads(line)["case"])
                    except (ValueError, KeyError):
                        continue  # a line cut short by an interrupted run: measured again
        else:
            if self.path.exists() or self.manifest_path.exists():
                raise ValueError(f"{self.path} exists: a fresh suite needs a new file (or resume it)")
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.manifest_path.write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
            self.path.touch()

    def write(self, row: dict) -> None:
        if row["case"] in self.done:
            raise ValueError(f"case {row['case']} is already recorded")
        with open(self.path, "a") as f:
            f.write(json.dumps(row) + "\n")
        self.done.add(row["case"])

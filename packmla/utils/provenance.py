"""Source identity, the source gate, and run manifests with SHA256SUMS.

    python -m packmla.utils.provenance sources [--strict]          print the identity; exit 1 if the gate fails
    python -m packmla.utils.provenance manifest RUN_DIR [-- CMD]   write manifest.json + SHA256SUMS for a run
    python -m packmla.utils.provenance verify RUN_DIR              recompute SHA256SUMS; exit 1 on a mismatch

Reference behaviour: scripts/sources.py (a read-only gate run before builds and host-side benchmarks that
pins the sources a compiled library was built from and fingerprints dirty trees) and benchmarks/README.md's
evidence rules (keep source/binary hashes, commands and raw measurements; verify checksums before curation;
never overwrite a saved run).  The gate here checks that the in-tree extension was built from the `csrc/` the
tree holds (the digest `setup.py` records beside the library) and, with `strict`, that no compiled source is
modified against the git commit.  A run directory is sealed by a manifest (source identity, software and
GPU, command) and a `SHA256SUMS` in `sha256sum` format covering every other file; sealing refuses a
directory that already has one.
"""
from __future__ import annotations

import argparse
import datetime as _dt
import hashlib
import json
import os
import platform
import subprocess
import sys
from pathlib import Path

from .source_digest import RECORD, source_digest

ROOT = Path(__file__).resolve().parents[2]
COMPILED_SUFFIXES = {".cu", ".cuh", ".cc", ".cpp", ".h", ".hpp", ".py"}


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _git(root: Path, *args: str) -> str | None:
    try:
        out = subprocess.run(["git", "-C", str(root), *args], capture_output=True, text=True, timeout=30)
    except (OSError, subprocess.SubprocessError):
        return None
    return out.stdout.rstrip("\n") if out.returncode == 0 else None


def source_identity(root: Path = ROOT) -> dict:
    """Commit, modified paths (with a digest of their current bytes), the compiled-source digest and the
    library's recorded build digest."""
    root = Path(root)
    commit = _git(root, "rev-parse", "HEAD")
    status = _git(root, "status", "--porcelain", "--untracked-files=no")
    dirty = sorted(line[3:] for line in status.splitlines()) if status else []
    h = hashlib.sha256()
    for rel in dirty:
        p = root / rel
        h.update(rel.encode() + b"\0" + (p.read_bytes() if p.is_file() else b"<deleted>") + b"\0")
    libs = sorted(root.glob("packmla/_C*.so"))
    recorded = None
    if (root / RECORD).exists():
        recorded = json.loads((root / RECORD).read_text()).get("sources_sha256")
    current = source_digest(str(root))
    return {
        "git_commit": commit,
        "modified": dirty,
        "modified_sha256": h.hexdigest() if dirty else None,
        "compiled_modified": [p for p in dirty if p.startswith("csrc/") or p == "setup.py"],
        "csrc_sha256": current,
        "library": {"path": str(libs[0].relative_to(root)) if libs else None,
                    "sha256": _sha256(libs[0]) if libs else None, "built_from_sha256": recorded},
        "library_matches_sources": recorded == current if recorded else None,
    }


def check_sources(root: Path = ROOT, strict: bool = False) -> dict:
    """The gate: raises RuntimeError when the built library does not match the sources (or is missing), and
    with `strict` when compiled sources differ from the commit; returns the identity otherwise."""
    ident = source_identity(root)
    if ident["library"]["path"] is None:
        raise RuntimeError("no built extension (packmla/_C*.so): run `python setup.py build_ext --inplace`")
    if ident["library_matches_sources"] is False:
        raise RuntimeError("the extension was built from other sources than csrc/ holds: rebuild it")
    if strict and ident["compiled_modified"]:
        raise RuntimeError("compiled sources differ from the commit: " + ", ".join(ident["compiled_modified"]))
    return ident


def environment() -> dict:
    out = {"python": platform.python_version(), "host": platform.node(), "platform": platform.platform()}
    try:
        import torch

        out["torch"] = torch.__version__
        out["cuda_runtime"] = torch.version.cuda
        if torch.cuda.is_available():
            out["gpus"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
    except ImportError:
        pass
    drv = None
    try:
        r = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"], capture_output=True,
                           text=True, timeout=20)
        drv = r.stdout.strip().splitlines()[0] if r.returncode == 0 and r.stdout.strip() else None
    except (OSError, subprocess.SubprocessError):
        pass
    out["driver"] = drv
    return out


def _files(run_dir: Path) -> list[Path]:
    return sorted(p for p in run_dir.rglob("*") if p.is_file() and p.name != "SHA256SUMS")


def write_sums(run_dir: Path) -> Path:
    run_dir = Path(run_dir)
    lines = [f"{_sha256(p)}  {p.relative_to(run_dir).as_posix()}" for p in _files(run_dir)]
    out = run_dir / "SHA256SUMS"
    out.write_text("\n".join(lines) + "\n")
    return out


def seal_run(run_dir: Path, command: list[str] | None = None, extra: dict | None = None,
             root: Path = ROOT) -> dict:
    """Write manifest.json and SHA256SUMS for a finished run directory (refuses a sealed one)."""
    run_dir = Path(run_dir)
    if not run_dir.is_dir():
        raise ValueError(f"run directory required: {run_dir}")
    if (run_dir / "SHA256SUMS").exists() or (run_dir / "manifest.json").exists():
        raise ValueError(f"run already sealed: {run_dir} (a changed protocol gets a new directory)")
    manifest = {"schema": "packmla-run-manifest-v1",
                "sealed_utc": _dt.datetime.now(_dt.timezone.utc).isoformat(timespec="seconds"),
                "command": command, "sources": source_identity(root), "environment": environment(),
                **({"extra": extra} if extra else {})}
    (run_dir / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    write_sums(run_dir)
    return manifest


def verify_run(run_dir: Path) -> list[str]:
    """Problems found (empty = the directory is exactly what its SHA256SUMS lists)."""
    run_dir = Path(run_dir)
    sums = run_dir / "SHA256SUMS"
    if not sums.exists():
        return ["no SHA256SUMS"]
    listed = {}
    for line in sums.read_text().splitlines():
        if line.strip():
            digest, rel = line.split("  ", 1)
            listed[rel] = digest
    problems = []
    present = {p.relative_to(run_dir).as_posix(): p for p in _files(run_dir)}
    for rel, digest in listed.items():
        if rel not in present:
            problems.append(f"missing: {rel}")
        elif _sha256(present[rel]) != digest:
            problems.append(f"changed: {rel}")
    problems += [f"unlisted: {rel}" for rel in sorted(set(present) - set(listed))]
    return problems


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("sources")
    s.add_argument("--strict", action="store_true", help="also refuse modified compiled sources")
    m = sub.add_parser("manifest")
    m.add_argument("run_dir", type=Path)
    m.add_argument("command", nargs=argparse.REMAINDER, help="the command that made the run (after --)")
    v = sub.add_parser("verify")
    v.add_argument("run_dir", type=Path)
    a = ap.parse_args(argv)
    if a.cmd == "sources":
        try:
            print(json.dumps(check_sources(strict=a.strict), indent=1))
            return 0
        except RuntimeError as e:
            print(f"source gate: {e}", file=sys.stderr)
            return 1
    if a.cmd == "manifest":
        cmd = [c for c in a.command if c != "--"] or None
        print(json.dumps(seal_run(a.run_dir, cmd), indent=1))
        return 0
    problems = verify_run(a.run_dir)
    print(json.dumps({"run": str(a.run_dir), "ok": not problems, "problems": problems}))
    return 0 if not problems else 1


if __name__ == "__main__":
    sys.exit(main())

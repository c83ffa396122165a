"""Which checks a change needs: maps the files a diff touches to a validation tier.

    python -m packmla.utils.validation_tier [--base main]          # files of `git diff --name-only base`
    python -m packmla.utils.validation_tier csrc/kv_store.cu ...   # explicit files

Reference behaviour: scripts/validation_tier.py maps a diff to low / medium / high required checks.
For packmla:

    high    device code or its bindings (csrc/, setup.py, the extension loader): rebuild for sm_100a,
            `pytest -m gpu` on a B200, the affected microbenchmark, an ncu capture of a changed kernel
    medium  Python that runs on the GPU path (ops, models, engine, KV pool, parallel, bench.py, the
            build entry): CPU tests, `pytest -m gpu`, a short `bench.py` run
    low     everything else (server, clients, training, formats oracle, docs, tests): CPU tests

The tier of a change is the highest tier of its files.
"""
from __future__ import annotations

import argparse
import fnmatch
import json
import subprocess

HIGH = ("csrc/*", "setup.py", "packmla/ops/_ext.py")
MEDIUM = ("packmla/ops/*", "packmla/models/*", "packmla/engine/*", "packmla/kv/*", "packmla/parallel/*",
          "bench.py", "__graft_entry__.py", "packmla/bench/microbench.py", "packmla/bench/synthetic.py",
          "packmla/bench/timing.py")
CHECKS = {
    "low": ["python -m pytest tests -m 'not gpu'"],
    "medium": ["python -m pytest tests -m 'not gpu'", "python -m pytest tests -m gpu (B200)",
               "python bench.py --steps 8 --warmup 3 (B200)"],
    "high": ["python setup.py build_ext --inplace", "python -m pytest tests -m 'not gpu'",
             "python -m pytest tests -m gpu (B200)", "python bench.py --steps 8 --warmup 3 (B200)",
             "the changed kernel's microbenchmark and one ncu capture on a small case (B200)"],
}
_ORDER = {"low": 0, "medium": 1, "high": 2}


def tier_of(path: str) -> str:
    if any(fnmatch.fnmatch(path, p) for p in HIGH):
        return "high"
    if any(fnmatch.fnmatch(path, p) for p in MEDIUM):
        return "medium"
    return "low"


def classify(paths: list[str]) -> dict:
    tiers = {p: tier_of(p) for p in paths}
    tier = max(tiers.values(), key=_ORDER.__getitem__, default="low")
    return {"tier": tier, "files": tiers, "required": CHECKS[tier]}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("files", nargs="*")
    ap.add_argument("--base", default=None, help="classify `git diff --name-only BASE` (with the work tree)")
    a = ap.parse_args(argv)
    files = list(a.files)
    if a.base is not None:
        files += subprocess.run(["git", "diff", "--name-only", a.base], capture_output=True, text=True,
                                check=True).stdout.split()
    out = classify(sorted(set(files)))
    print(json.dumps(out, indent=2))
    return out


if __name__ == "__main__":
    main()

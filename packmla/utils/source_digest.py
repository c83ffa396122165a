"""Digest of the sources the CUDA extension is built from, recorded beside the library at build time.

The extension is built in-tree and travels with the checkout, so a library built from older sources
can outlive an edit of `csrc/`.  `setup.py` writes `packmla/_C.sources.json` after every build;
`packmla.ops._ext` compares it with the current sources when it loads the library and warns on a
mismatch.  Reference behaviour: scripts/sources.py `compiled_source_digest`, which pins the sources
a compiled image was built from.
"""
from __future__ import annotations

import glob
import hashlib
import json
import os

RECORD = os.path.join("packmla", "_C.sources.json")


def source_digest(root: str) -> str:
    """sha256 over the relative paths and contents of csrc/ (recursively) and setup.py."""
    files = sorted(glob.glob(os.path.join(root, "csrc", "**", "*"), recursive=True)) + [os.path.join(root, "setup.py")]
    h = hashlib.sha256()
    for path in files:
        if os.path.isfile(path):
            h.update(os.path.relpath(path, root).replace(os.sep, "/").encode() + b"\0")
            with open(path, "rb") as f:
                h.update(f.read())
            h.update(b"\0")
    return h.hexdigest()


def write_record(root: str) -> str:
    digest = source_digest(root)
    with open(os.path.join(root, RECORD), "w") as f:
        json.dump({"sources_sha256": digest}, f)
    return digest


def check_record(root: str) -> str | None:
    """None when the record matches the sources (or there is no record); else a message."""
    path = os.path.join(root, RECORD)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        recorded = json.load(f).get("sources_sha256")
    if recorded != source_digest(root):
        return "packmla/_C was built from different sources than csrc/ now holds: rebuild with " \
               "`python setup.py build_ext --inplace`"
    return None

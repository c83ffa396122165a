"""Exclusive lock around in-tree extension builds.

Two builds writing `packmla/_C*.so` at once can leave a torn library behind, which the next import
loads.  `build_lock()` takes an exclusive `flock` on `build/.packmla-build.lock` (released by the
kernel when the holder exits, so a crashed build leaves no stale lock) and records the holder's pid
and start time in the file for the error message of a build that waits too long.  Reference
behaviour: scripts/build_lock.py (a lock file with pid / start-time liveness checks).
"""
from __future__ import annotations

import contextlib
import fcntl
import json
import os
import time


class BuildLocked(RuntimeError):
    pass


@contextlib.contextmanager
def build_lock(root: str, timeout_s: float = 600.0, poll_s: float = 0.5):
    os.makedirs(os.path.join(root, "build"), exist_ok=True)
    path = os.path.join(root, "build", ".packmla-build.lock")
    f = open(path, "a+")
    try:
        deadline = time.monotonic() + timeout_s
        while True:
            try:
                fcntl.flock(f.fileno(), fcntl.LOCK_EX | fcntl.LOCK_NB)
                break
            except BlockingIOError:
                if time.monotonic() >= deadline:
                    f.seek(0)
                    holder = f.read().strip() or "unknown holder"
                    raise BuildLocked(f"another build holds {path}: {holder}") from None
                time.sleep(poll_s)
        f.seek(0)
        f.truncate()
        f.write(json.dumps({"pid": os.getpid(), "started": time.time()}))
        f.flush()
        yield path
    finally:
        f.close()  # closing the descriptor releases the lock

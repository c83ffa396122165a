"""Deadline-bounded capture launcher: one capture run in its own process group, with owned clean-up.

    python -m packmla.training.data.capture_launch --deadline 3600 -- --output cache/ --model small --issues 32

Reference behaviour: scripts/local/capture-latent.sh, which runs the latent capture in an isolated Native
serving container under deadlines and removes what it started on every exit path.  packmla's capture runs
its own Native-mode engine (packmla.training.data.capture), so the launcher owns that process instead:

  * the capture runs in a new session, writing into a staging directory beside the requested output
    (`<output>.staging-<pid>`), never into the output itself;
  * exit 0 within the deadline: the staging directory is renamed to the output (which must not exist);
  * failure, deadline or interrupt: the child's process group alone is signalled (SIGTERM, then SIGKILL
    after a grace period), the staging directory is removed, and the launcher exits non-zero;
  * `<output>.launch.json` records the command, the outcome, the exit code and the seconds taken.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import signal
import subprocess
import sys
import time
from pathlib import Path


def _stop_group(proc: subprocess.Popen, grace_s: float) -> None:
    try:
        os.killpg(proc.pid, signal.SIGTERM)
    except ProcessLookupError:
        return
    try:
        proc.wait(grace_s)
    except subprocess.TimeoutExpired:
        try:
            os.killpg(proc.pid, signal.SIGKILL)
        except ProcessLookupError:
            pass
        proc.wait(grace_s)


def launch(capture_args: list[str], deadline_s: float, grace_s: float = 30.0,
           command: list[str] | None = None) -> dict:
    """Run one capture under a deadline.  `command` replaces the capture module (tests); "{output}" in it
    stands for the staging directory."""
    if "--output" not in capture_args:
        raise ValueError("the capture arguments need --output")
    i = capture_args.index("--output")
    output = Path(capture_args[i + 1])
    if output.exists():
        raise ValueError(f"fresh output directory required: {output}")
    staging = output.with_name(f"{output.name}.staging-{os.getpid()}")
    args = list(capture_args)
    args[i + 1] = str(staging)
    cmd = ([c.replace("{output}", str(staging)) for c in command] if command
           else [sys.executable, "-m", "packmla.training.data.capture"] + args)
    record = {"command": cmd, "output": str(output), "deadline_s": deadline_s}
    t0 = time.monotonic()
    proc = subprocess.Popen(cmd, start_new_session=True)
    prev = {}

    def on_signal(signum, frame):
        raise KeyboardInterrupt

    for s in (signal.SIGINT, signal.SIGTERM):
        prev[s] = signal.signal(s, on_signal)
    try:
        try:
            rc = proc.wait(timeout=deadline_s)
            outcome = "completed" if rc == 0 else "failed"
        except subprocess.TimeoutExpired:
            _stop_group(proc, grace_s)
            rc, outcome = proc.returncode, "deadline"
    except KeyboardInterrupt:
        _stop_group(proc, grace_s)
        rc, outcome = proc.returncode, "interrupted"
    finally:
        for s, h in prev.items():
            signal.signal(s, h)
    if outcome == "completed" and staging.is_dir():
        os.rename(staging, output)
    else:
        if outcome == "completed":
            outcome = "failed"  # exited 0 without writing its output
        shutil.rmtree(staging, ignore_errors=True)
    record.update(outcome=outcome, exit_code=rc, seconds=round(time.monotonic() - t0, 2))
    output.with_name(output.name + ".launch.json").write_text(json.dumps(record, indent=1) + "\n")
    return record


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--" not in argv:
        raise SystemExit("usage: capture_launch [--deadline S] [--grace S] -- <capture arguments>")
    k = argv.index("--")
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--deadline", type=float, default=3600.0)
    ap.add_argument("--grace", type=float, default=30.0)
    a = ap.parse_args(argv[:k])
    rec = launch(argv[k + 1:], a.deadline, a.grace)
    print(json.dumps(rec))
    return 0 if rec["outcome"] == "completed" else 1


if __name__ == "__main__":
    sys.exit(main())

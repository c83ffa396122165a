"""Environment report and server helpers for a serving or benchmark host.

    python -m packmla.utils.env report                # software, GPUs, clocks, NVLink topology, NCCL settings
    python -m packmla.utils.env health [URL]          # exit 0 when the server answers /health with "ok"
    python -m packmla.utils.env pool [URL]            # the server's KV pool (/server_info) as JSON
    python -m packmla.utils.env kill-port PORT        # stop the one process listening on PORT (exact PID)

Reference behaviour: scripts/local/env.sh (machine configuration and the `health`, `kill_port`, `pool_of`
helpers) and scripts/local/container.sh's image verification.  packmla runs in the image it was built in,
so the report records what a run depends on instead of building a container: Python, torch, CUDA and
NCCL versions, the in-tree extension's identity, every GPU with its clocks and throttle reasons (read
only), the NVLink topology matrix and the NCCL_* environment.  `kill_port` signals only the process that
owns the listening socket (SIGTERM, then SIGKILL after a grace period), never a name pattern.
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys

DEFAULT_URL = "http://127.0.0.1:30000"
GPU_FIELDS = ("index", "name", "memory.total", "clocks.sm", "clocks.max.sm", "power.draw", "power.limit",
              "clocks_event_reasons.active")


def _run(cmd: list[str], timeout: float = 30.0) -> str | None:
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    except (OSError, subprocess.SubprocessError):
        return None
    return out.stdout if out.returncode == 0 else None


def gpus() -> list[dict]:
    """One dict per GPU from nvidia-smi's query interface (read only); [] without a GPU."""
    out = _run(["nvidia-smi", f"--query-gpu={','.join(GPU_FIELDS)}", "--format=csv,noheader,nounits"])
    if not out:
        return []
    rows = []
    for line in out.strip().splitlines():
        vals = [v.strip() for v in line.split(",")]
        rows.append(dict(zip(GPU_FIELDS, vals)))
    return rows


def report() -> dict:
    from .provenance import environment, source_identity

    out = {"environment": environment(), "gpus": gpus(),
           "nvlink_topology": _run(["nvidia-smi", "topo", "-m"]),
           "nccl_env": {k: v for k, v in sorted(os.environ.items()) if k.startswith("NCCL_")}}
    try:
        import torch

        out["nccl_version"] = ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None
    except (ImportError, AttributeError, RuntimeError):
        out["nccl_version"] = None
    ident = source_identity()
    out["extension"] = {"library": ident["library"], "matches_sources": ident["library_matches_sources"],
                        "git_commit": ident["git_commit"]}
    return out


def health(url: str = DEFAULT_URL, timeout: float = 3.0) -> bool:
    import requests

    try:
        r = requests.get(url.rstrip("/") + "/health", timeout=timeout)
    except requests.RequestException:
        return False
    return r.status_code == 200 and r.text.strip() == "ok"


def pool_of(url: str = DEFAULT_URL, timeout: float = 10.0) -> dict:
    """The KV pool fields of the server's /server_info."""
    import requests

    info = requests.get(url.rstrip("/") + "/server_info", timeout=timeout).json()
    keys = ("kv_cache_format", "max_total_num_tokens", "bytes_per_full_token", "num_pages", "context_length",
            "max_running_requests", "tp", "prefix_cache", "prefix_blocks", "enable_hierarchical_cache")
    return {k: info.get(k) for k in keys if k in info}


def listener_pid(port: int) -> int | None:
    """PID of the process with a listening TCP socket on `port` (None if none is found)."""
    import psutil

    for c in psutil.net_connections(kind="tcp"):
        if c.laddr and c.laddr.port == port and c.status == psutil.CONN_LISTEN and c.pid:
            return c.pid
    return None


def kill_port(port: int, grace_s: float = 10.0) -> int | None:
    """Stop the process listening on `port`: SIGTERM, then SIGKILL after `grace_s`.  Returns its PID."""
    import psutil

    pid = listener_pid(port)
    if pid is None or pid == os.getpid():
        return None
    proc = psutil.Process(pid)
    proc.send_signal(signal.SIGTERM)
    try:
        proc.wait(grace_s)
    except psutil.TimeoutExpired:
        proc.kill()
        proc.wait(grace_s)
    return pid


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("report")
    h = sub.add_parser("health")
    h.add_argument("url", nargs="?", default=DEFAULT_URL)
    p = sub.add_parser("pool")
    p.add_argument("url", nargs="?", default=DEFAULT_URL)
    k = sub.add_parser("kill-port")
    k.add_argument("port", type=int)
    k.add_argument("--grace", type=float, default=10.0)
    a = ap.parse_args(argv)
    if a.cmd == "report":
        print(json.dumps(report(), indent=1))
        return 0
    if a.cmd == "health":
        ok = health(a.url)
        print("ok" if ok else "unhealthy")
        return 0 if ok else 1
    if a.cmd == "pool":
        print(json.dumps(pool_of(a.url)))
        return 0
    pid = kill_port(a.port, a.grace)
    print(json.dumps({"port": a.port, "stopped_pid": pid}))
    return 0 if pid is not None else 1


if __name__ == "__main__":
    sys.exit(main())

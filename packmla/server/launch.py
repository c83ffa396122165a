"""Environment-driven server launcher: the counterpart of the reference's scripts/local/serve.sh and
run-server.sh (settings as named environment values, scripts/local/launch-config.sh:44-54).

    TP=4 PORT=30000 MEM_FRAC=0.88 python -m packmla.server.launch direct
    MODEL=tiny DEVICE=cpu python -m packmla.server.launch native --smoke     # start, wait, read out, stop
    TP=8 python -m packmla.server.launch direct --dry-run                   # print the command only

Environment (all optional): MODE (native | direct; the positional mode wins), MODEL_FAMILY (dsv4 | dsv41 |
glm53; dsv41 serves the V4.1 FP4 cache formats), MODEL (default v4-flash),
DEVICE (cuda | cpu), TP, EP, PORT (30000), MASTER_PORT (29500), MEM_FRAC, CTX_LEN, MAX_RUN, CHUNK,
DECODE_CFG (the --cuda-graph-config JSON), SERVER_SEED, HICACHE_RATIO (turns HiCache on),
C4_KEEP_COUNT, C4_LAYER_KEEP_COUNTS, STORE_IMPLEMENTATION, REQUEST_METRICS_DIR (request log and
per-request metric files; the directory must exist), DSV4_ASYNC_PREPARATION (0 | 1) and
DSV4_PREPARATION_WORKERS (1 | 2 | 4): chat conversion off the API loop, FRONTEND_DIAGNOSTICS (0 | 1),
NSYS_OUTPUT (run under Nsight Systems, which records only between POST /start_profile and /stop_profile).  TP > 1 runs one process per GPU under torchrun
on 127.0.0.1.

The launcher owns the server's process group: it starts the server in a new session, waits for
`/health` (bounded by --wait-timeout, failing early if the server exits), prints one JSON line with
the pool read out of `/server_info`, and on exit, SIGINT or SIGTERM stops the whole group (SIGTERM,
then SIGKILL after a grace period).  Only that group is signalled.
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import signal
import subprocess
import sys
import time

ENV_FLAGS = (  # environment name -> server flag
    ("TP", "--tp"), ("EP", "--ep"), ("MEM_FRAC", "--mem-fraction-static"), ("CTX_LEN", "--context-length"),
    ("MAX_RUN", "--max-running-requests"), ("CHUNK", "--chunked-prefill-size"),
    ("DECODE_CFG", "--cuda-graph-config"), ("SERVER_SEED", "--random-seed"),
    ("C4_KEEP_COUNT", "--dsv4-c4-cache-keep-count"), ("C4_LAYER_KEEP_COUNTS", "--dsv4-c4-cache-layer-keep-counts"),
    ("STORE_IMPLEMENTATION", "--dsv4-c4-cache-store-implementation"),
)


FAMILIES = ("dsv4", "dsv41", "glm53")
CODEC_OVERRIDES = ("HICACHE_RATIO", "C4_KEEP_COUNT", "C4_LAYER_KEEP_COUNTS", "STORE_IMPLEMENTATION")


def _family_checks(family: str, env: dict) -> tuple[int, int | None]:
    """(TP, EP) of a V4.1 or GLM-5.3 launch, validated as the reference's launch configuration does
    (scripts/local/launch-config.sh:10-38, run-server.sh:82-97): TP 1, 2, 4 or 8; EP (default TP) a
    divisor of TP; no HiCache or C4 codec overrides; an explicit GPU list names exactly TP devices."""
    label = "V4.1" if family == "dsv41" else "GLM"
    tp = int(env.get("TP", "4" if family == "dsv41" else "8"))
    if tp not in (1, 2, 4, 8):
        raise SystemExit(f"{label} launches take a TP size of 1, 2, 4 or 8 (got {tp})")
    ep = int(env.get("EP", str(tp)))
    if ep < 1 or ep > tp or tp % ep:
        raise SystemExit(f"{label}: EP={ep} does not divide TP={tp}")
    if any(env.get(k) for k in CODEC_OVERRIDES):
        raise SystemExit(f"{label}: HiCache and the C4 codec settings ({', '.join(CODEC_OVERRIDES)}) apply to dsv4 "
                         "only")
    gpus = env.get("GPUS") or env.get("CUDA_VISIBLE_DEVICES")
    if gpus:
        devices = gpus.split(",")
        if len(devices) != tp or any(not d.strip() for d in devices):
            raise SystemExit(f"{label}: the GPU list {gpus!r} must name exactly {tp} devices")
    return tp, ep


def resolve(mode: str | None, env: dict) -> tuple[list[str], dict]:
    """(command, extra environment) of the server launch described by `env`.  MODEL_FAMILY selects dsv4
    (default), dsv41 (the V4.1 FP4 cache: native -> fp4-native, direct -> fp4-direct, EP ranks) or glm53."""
    mode = mode or env.get("MODE", "direct")
    if mode not in ("native", "direct"):
        raise SystemExit(f"mode must be native or direct, not {mode!r}")
    family = env.get("MODEL_FAMILY", "dsv4")
    if family not in FAMILIES:
        raise SystemExit(f"unknown MODEL_FAMILY {family!r} (one of {', '.join(FAMILIES)})")
    fmt = mode
    if family != "dsv4":
        tp, ep = _family_checks(family, env)
        if family == "glm53":
            raise SystemExit("GLM-5.3 serving is not built: packmla provides the GLM MLA row formats, stores, "
                             "Adapter and decode (packmla.ops.glm, packmla.kv.glm_pool), not the GLM model "
                             "(KDA layers, hyper-connections)")
        if ep != tp:
            raise SystemExit(f"EP={ep}: packmla shards the routed experts over the TP ranks (EP = TP = {tp})")
        env = {**env, "TP": str(tp), "EP": str(ep)}
        fmt = "fp4-" + mode
    tp = int(env.get("TP", "1"))
    if tp < 1:
        raise SystemExit("TP must be >= 1")
    port = env.get("PORT", "30000")
    flags = ["--model", env.get("MODEL", "v4-flash"), "--kv-cache-format", fmt, "--port", port,
             "--device", env.get("DEVICE", "cuda")]
    for name, flag in ENV_FLAGS:
        if env.get(name):
            flags += [flag, env[name]]
    diag = env.get("FRONTEND_DIAGNOSTICS", "0")
    if diag not in ("0", "1"):
        raise SystemExit(f"FRONTEND_DIAGNOSTICS takes 0 or 1, not {diag!r}")
    prep = env.get("DSV4_ASYNC_PREPARATION", "0")
    if prep not in ("0", "1"):
        raise SystemExit(f"DSV4_ASYNC_PREPARATION takes 0 or 1, not {prep!r}")
    workers = env.get("DSV4_PREPARATION_WORKERS", "1")
    if workers not in ("1", "2", "4"):
        raise SystemExit(f"DSV4_PREPARATION_WORKERS takes 1, 2 or 4, not {workers!r}")
    # the reference launches serve the DeepSeek families with their reasoning parser
    flags += ["--reasoning-parser", "deepseek-v41" if family == "dsv41" else "deepseek-v4"]
    if prep == "1":
        flags += ["--chat-preparation-workers", workers]
    if diag == "1":
        flags += ["--frontend-diagnostics"]
    if env.get("HICACHE_RATIO"):
        flags += ["--enable-hierarchical-cache", "--hicache-ratio", env["HICACHE_RATIO"]]
    metrics_dir = env.get("REQUEST_METRICS_DIR")
    if metrics_dir:
        if not os.path.isdir(metrics_dir):
            raise SystemExit(f"request metrics directory does not exist: {metrics_dir}")
        flags += ["--enable-metrics", "--log-requests", "--log-requests-level", "0", "--export-metrics-to-file",
                  "--export-metrics-to-file-dir", metrics_dir]
    if tp > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(tp),
               "--master-addr", "127.0.0.1", "--master-port", env.get("MASTER_PORT", "29500"),
               "-m", "packmla.server"]
    else:
        cmd = [sys.executable, "-m", "packmla.server"]
    if env.get("NSYS_OUTPUT"):  # Nsight Systems attached at launch, collecting between /start_profile and /stop_profile
        import shutil

        nsys = shutil.which("nsys", path=env.get("PATH"))
        if nsys is None:
            raise SystemExit("NSYS_OUTPUT is set but nsys is not on PATH")
        cmd = [nsys, "profile", "-o", env["NSYS_OUTPUT"], "--trace=cuda,nvtx", "--capture-range=cudaProfilerApi",
               "--capture-range-end=stop", "--force-overwrite=false"] + cmd
    extra = {"NCCL_SOCKET_IFNAME": env.get("NCCL_SOCKET_IFNAME", "lo"),
             "GLOO_SOCKET_IFNAME": env.get("GLOO_SOCKET_IFNAME", "lo")}
    return cmd + flags, extra


class ServerGroup:
    """A server process started in its own session; `stop()` signals exactly that process group."""

    def __init__(self, cmd: list[str], env: dict, log_path: str | None = None):
        self.log = open(log_path, "ab") if log_path else None
        self.proc = subprocess.Popen(cmd, env=env, start_new_session=True,
                                     stdout=self.log or None, stderr=subprocess.STDOUT if self.log else None)
        self.pgid = os.getpgid(self.proc.pid)

    def alive(self) -> bool:
        return self.proc.poll() is None

    def stop(self, grace_s: float = 30.0) -> int:
        if self.alive():
            try:
                os.killpg(self.pgid, signal.SIGTERM)
            except ProcessLookupError:
                pass
            try:
                self.proc.wait(grace_s)
            except subprocess.TimeoutExpired:
                try:
                    os.killpg(self.pgid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
                self.proc.wait(10)
        if self.log:
            self.log.close()
        return self.proc.returncode


def wait_ready(url: str, group: ServerGroup, timeout_s: float) -> dict:
    """Poll /health until 200; returns /server_info.  Raises if the server exits or the time runs out."""
    import requests

    deadline = time.monotonic() + timeout_s
    while time.monotonic() < deadline:
        if not group.alive():
            raise RuntimeError(f"server exited with code {group.proc.returncode} before it was healthy")
        try:
            if requests.get(url + "/health", timeout=5).status_code == 200:
                from ..bench.serving import auth_headers

                return requests.get(url + "/server_info", timeout=30, headers=auth_headers()).json()
        except requests.RequestException:
            pass
        time.sleep(0.5)
    raise RuntimeError(f"server not healthy within {timeout_s} s")


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("mode", nargs="?", choices=["native", "direct"], default=None)
    ap.add_argument("--dry-run", action="store_true", help="print the resolved command and exit")
    ap.add_argument("--smoke", action="store_true", help="start, wait for health, read the pool out, stop")
    ap.add_argument("--wait-timeout", type=float, default=1800.0)
    ap.add_argument("--log", default=None, help="append the server's output to this file")
    a = ap.parse_args(argv)
    cmd, extra = resolve(a.mode, dict(os.environ))
    if a.dry_run:
        out = {"command": shlex.join(cmd), "env": extra}
        print(json.dumps(out))
        return out
    env = dict(os.environ)
    env.update(extra)
    group = ServerGroup(cmd, env, a.log)
    if not a.smoke:  # foreground: a signal to the launcher stops the server group
        def on_signal(signum, frame):
            group.stop()
            raise SystemExit(128 + signum)

        signal.signal(signal.SIGTERM, on_signal)
        signal.signal(signal.SIGINT, on_signal)
    url = f"http://127.0.0.1:{os.environ.get('PORT', '30000')}"
    try:
        info = wait_ready(url, group, a.wait_timeout)
        out = {"event": "ready", "url": url, "pgid": group.pgid,
               **{k: info.get(k) for k in ("kv_cache_format", "max_total_num_tokens", "bytes_per_full_token",
                                           "max_running_requests", "context_length", "tp", "prefix_cache",
                                           "enable_hierarchical_cache")}}
        print(json.dumps(out), flush=True)
        if a.smoke:
            return out
        group.proc.wait()
        return out
    finally:
        group.stop()


if __name__ == "__main__":
    main()

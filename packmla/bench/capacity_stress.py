"""Multi-turn capacity stress with the KV reuse tiers on and off (one server per setting).

    TP=4 python -m packmla.bench.capacity_stress direct --sessions 64 --turns 4 --input-len 8192 \
        --output-len 256 --concurrency 32 [--settings none,hicache,prefix,both]

Each setting starts its own server through `packmla.server.launch` (the environment's settings, plus
the setting's cache flags), runs the multi-turn dataset of `packmla.bench.serving` (every session
re-sends its growing history each turn, so later turns can reuse earlier turns' KV), reads the
server's reuse counters from `/metrics`, and stops the server.  Settings:

    none      --disable-radix-cache, no HiCache: every turn prefills its whole history
    hicache   host tier only (HICACHE_RATIO, default 2): finished turns restored from pinned host memory
    prefix    device prefix cache only: finished turns kept on the device while space allows
    both      device prefix cache first, host tier behind it

The result gives per setting and turn the TTFT and throughput, and the tokens each tier saved.
Reference: its multi-turn capacity experiments with HiCache on and off at fixed pool size
(scripts/local/README.md "CPU-L2 HiCache screening").
"""
from __future__ import annotations

import argparse
import json
import os

SETTINGS = {"none": {"radix": False, "hicache": False}, "hicache": {"radix": False, "hicache": True},
            "prefix": {"radix": True, "hicache": False}, "both": {"radix": True, "hicache": True}}


def _metric(url: str, name: str) -> float:
    import requests

    from .serving import auth_headers

    for line in requests.get(url + "/metrics", timeout=30, headers=auth_headers()).text.splitlines():
        if line.startswith(f"packmla_{name} "):
            return float(line.split()[1])
    return 0.0


def run_setting(mode: str, setting: str, *, sessions: int, turns: int, input_len: int, output_len: int,
                concurrency: int, startup_timeout_s: float = 1800.0, log_dir: str | None = None) -> dict:
    from ..server import launch
    from .serving import bench

    env = dict(os.environ)
    s = SETTINGS[setting]
    if s["hicache"]:
        env.setdefault("HICACHE_RATIO", "2")
    else:
        env.pop("HICACHE_RATIO", None)
    cmd, extra = launch.resolve(mode, env)
    if not s["radix"]:
        cmd.append("--disable-radix-cache")
    env.update(extra)
    group = launch.ServerGroup(cmd, env, os.path.join(log_dir, f"{setting}.server.log") if log_dir else None)
    url = f"http://127.0.0.1:{env.get('PORT', '30000')}"
    try:
        info = launch.wait_ready(url, group, startup_timeout_s)
        out = bench(url, "multi-turn", input_len, output_len, concurrency, flush_cache=True, turns=turns,
                    sessions=sessions)
        return {"setting": setting, "max_total_num_tokens": info.get("max_total_num_tokens"),
                "turns": [{k: t[k] for k in ("completed", "success_rate", "output_throughput_tok_s", "ttft_ms",
                                             "validated")} for t in out["turns"]],
                "prefix_cache_hit_tokens": _metric(url, "prefix_cache_hit_tokens"),
                "hicache_hit_tokens": _metric(url, "hicache_hit_tokens"),
                "prefill_tokens": _metric(url, "prefill_tokens")}
    finally:
        group.stop()


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("mode", choices=["native", "direct"])
    ap.add_argument("--settings", default="none,hicache,prefix,both")
    ap.add_argument("--sessions", type=int, default=16)
    ap.add_argument("--turns", type=int, default=4)
    ap.add_argument("--input-len", type=int, default=8192)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--concurrency", type=int, default=16)
    ap.add_argument("--startup-timeout", type=float, default=1800.0)
    ap.add_argument("--log-dir", default=None)
    ap.add_argument("--output", default=None, help="also write the result here (a new file)")
    a = ap.parse_args(argv)
    names = [x for x in a.settings.split(",") if x]
    bad = [x for x in names if x not in SETTINGS]
    if bad:
        raise SystemExit(f"unknown settings {bad}; choose from {sorted(SETTINGS)}")
    if a.log_dir:
        os.makedirs(a.log_dir, exist_ok=True)
    out = {"mode": a.mode, "sessions": a.sessions, "turns": a.turns, "input_len": a.input_len,
           "output_len": a.output_len, "concurrency": a.concurrency,
           "results": [run_setting(a.mode, n, sessions=a.sessions, turns=a.turns, input_len=a.input_len,
                                   output_len=a.output_len, concurrency=a.concurrency,
                                   startup_timeout_s=a.startup_timeout, log_dir=a.log_dir) for n in names]}
    text = json.dumps(out, indent=2)
    if a.output:
        with open(a.output, "x") as f:
            f.write(text)
    print(text)
    return out


if __name__ == "__main__":
    main()

"""Replay of recorded multi-turn sessions against an OpenAI-compatible server, fixed active-user pool.

    python -m packmla.bench.replay --base-url http://127.0.0.1:30000 --requests sessions.jsonl \
        --users 24 [--min-success 0.99] [--output summary.json]

Reference behaviour (the reference's LongSWE replay, scripts/local/business_replay/runner.py): a fixed
pool of active users; each user takes the next unreplayed session and sends its turns in order
(a turn starts when the previous one finished), every turn as a streamed chat completion; the run
reports per-request TTFT / E2E, output throughput, and fails its gate when fewer than `min_success` of
the requests complete.  Input: one JSON object per line,

    {"session": "s1", "turn": 0, "messages": [{"role": "user", "content": "..."}], "max_tokens": 256}

The summary also reports the server's HiCache restored-token counter delta (from /metrics), the share
of prompt work that a host-tier restore saved.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import time
from collections import defaultdict

import numpy as np


def load_sessions(path: str) -> list[list[dict]]:
    """JSONL -> sessions (lists of turns in turn order), sessions in first-appearance order."""
    sessions: dict[str, list[dict]] = defaultdict(list)
    order: list[str] = []
    with open(path) as f:
        for n, line in enumerate(f, 1):
            if not line.strip():
                continue
            rec = json.loads(line)
            if not isinstance(rec.get("messages"), list) or "session" not in rec:
                raise ValueError(f"line {n}: session and messages required")
            sid = str(rec["session"])
            if sid not in sessions:
                order.append(sid)
            sessions[sid].append(rec)
    return [sorted(sessions[s], key=lambda r: r.get("turn", 0)) for s in order]


async def _turn(session, url: str, model: str, rec: dict) -> dict:
    body = {"model": model, "messages": rec["messages"], "max_tokens": int(rec.get("max_tokens", 256)),
            "temperature": float(rec.get("temperature", 0.0)), "stream": True,
            "ignore_eos": bool(rec.get("ignore_eos", True))}
    t0 = time.perf_counter()
    out = {"session": str(rec["session"]), "turn": rec.get("turn", 0), "ok": False, "ttft": None, "tokens": 0}
    try:
        async with session.post(url + "/v1/chat/completions", json=body) as resp:
            if resp.status != 200:
                out["error"] = f"HTTP {resp.status}"
                return out
            async for raw in resp.content:
                line = raw.decode().strip()
                if not line.startswith("data: ") or line == "data: [DONE]":
                    continue
                delta = json.loads(line[6:])["choices"][0]
                if delta.get("delta", {}).get("content"):
                    if out["ttft"] is None:
                        out["ttft"] = time.perf_counter() - t0
                    out["tokens"] += 1
                if delta.get("finish_reason") in ("length", "stop"):
                    out["ok"] = True
    except Exception as exc:  # network failures count against the success gate
        out["error"] = repr(exc)
    out["e2e"] = time.perf_counter() - t0
    return out


async def _replay(url: str, model: str, sessions: list[list[dict]], users: int) -> tuple[list[dict], float]:
    import aiohttp

    queue: asyncio.Queue = asyncio.Queue()
    for s in sessions:
        queue.put_nowait(s)
    results: list[dict] = []
    timeout = aiohttp.ClientTimeout(total=None, sock_read=3600)
    async with aiohttp.ClientSession(timeout=timeout) as http:
        async def user():
            while True:
                try:
                    turns = queue.get_nowait()
                except asyncio.QueueEmpty:
                    return
                for rec in turns:  # a session's turns run in order
                    results.append(await _turn(http, url, model, rec))

        t0 = time.perf_counter()
        await asyncio.gather(*(user() for _ in range(max(1, users))))
        return results, time.perf_counter() - t0


def _metric(url: str, name: str) -> float:
    import requests

    try:
        for line in requests.get(url + "/metrics", timeout=30).text.splitlines():
            if line.startswith(name + " "):
                return float(line.split()[1])
    except requests.RequestException:
        pass
    return 0.0


def replay(url: str, requests_path: str, users: int, model: str = "default", min_success: float = 0.99) -> dict:
    sessions = load_sessions(requests_path)
    hits0 = _metric(url, "packmla_hicache_hit_tokens")
    results, wall = asyncio.run(_replay(url, model, sessions, users))
    ok = [r for r in results if r["ok"]]

    def pct(xs, q):
        return float(np.percentile(np.asarray(xs) * 1000, q)) if xs else None

    ttft = [r["ttft"] for r in ok if r["ttft"] is not None]
    e2e = [r["e2e"] for r in ok]
    success = len(ok) / max(1, len(results))
    return {"sessions": len(sessions), "requests": len(results), "completed": len(ok), "success_rate": success,
            "passed": success >= min_success, "users": users, "wall_s": wall,
            "output_tokens": sum(r["tokens"] for r in ok),
            "output_throughput_tok_s": sum(r["tokens"] for r in ok) / wall if wall > 0 else 0.0,
            "ttft_ms": {"p50": pct(ttft, 50), "p99": pct(ttft, 99)}, "e2e_ms": {"p50": pct(e2e, 50), "p99": pct(e2e, 99)},
            "hicache_restored_tokens": _metric(url, "packmla_hicache_hit_tokens") - hits0,
            "errors": [r.get("error") for r in results if not r["ok"]][:5]}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--base-url", default="http://127.0.0.1:30000")
    ap.add_argument("--requests", required=True)
    ap.add_argument("--users", type=int, default=24)
    ap.add_argument("--model", default="default")
    ap.add_argument("--min-success", type=float, default=0.99)
    ap.add_argument("--output", default=None)
    a = ap.parse_args(argv)
    out = replay(a.base_url, a.requests, a.users, a.model, a.min_success)
    text = json.dumps(out, indent=2)
    if a.output:
        with open(a.output, "x") as f:
            f.write(text)
    print(text)
    if not out["passed"]:
        raise SystemExit(f"success rate {out['success_rate']:.4f} below {a.min_success}")
    return out


if __name__ == "__main__":
    main()

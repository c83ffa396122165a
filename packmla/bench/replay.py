"""Replay of recorded multi-turn sessions against an OpenAI-compatible server, fixed active-user pool.

    python -m packmla.bench.replay --base-url http://127.0.0.1:30000 --requests sessions.jsonl \
        --users 24 [--min-success 0.99] [--duration-s 1200] [--ttft-slo-ms 10000] [--output summary.json]
    python -m packmla.bench.replay sweep --requests sessions.jsonl --concurrencies 20,22,24 \
        --repeats 1 --duration-s 1200 --out-dir results/sweep-direct
    python -m packmla.bench.replay plan --requests sessions.jsonl --pool-tokens 800512 --concurrencies 16,20,24

Reference behaviour (the reference's LongSWE replay, scripts/local/business_replay/runner.py): a fixed
pool of active users; each user takes the next unreplayed session and sends its turns in order
(a turn starts when the previous one finished), every turn as a streamed chat completion; the run
reports per-request TTFT / E2E, output throughput, and fails its gate when fewer than `min_success` of
the requests complete.  Input: one JSON object per line,

    {"session": "s1", "turn": 0, "messages": [{"role": "user", "content": "..."}], "max_tokens": 256}

The summary also reports the server's HiCache restored-token counter delta (from /metrics), the share
of prompt work that a host-tier restore saved.

`--duration-s` is the dispatch window: after it no user starts a new session, sessions already
started finish (the drain), and rates divide by the whole wall time, drain included.  Completeness
(every started session finished), response success (>= `min_success`, inclusive) and TTFT p90
(strictly below `ttft_slo_ms`) are separate fields; `passed` needs all three.

`sweep` (reference: scripts/local/sweep-lswb.sh, scripts/local/business_replay/sweep.py) replays one
running server at an ordered ladder of concurrencies, `repeats` consecutive replays per point, each
after the server is idle and its cache flushed.  Every point's summary lands in
`<out-dir>/c<N>/repeat-<NN>/summary.json` and the incremental `summary.json` / `summary.csv`; a failed
gate is recorded and later points still run, while an unhealthy server or a failed flush stops the
sweep.  No best point is chosen.

`--scheduler request-slot` replays the closed-loop request-slot FIFO (`request_slot_replay`): a fixed
window, throughput inside it, and a queue-inclusive ready-to-first-output SLO.

`plan` (reference: scripts/local/business_replay/capacity_plan.py) replays the scheduler offline: C
slots each hold one session and send its requests one per tick; the live context of a tick is the
sum of the active requests' sizes (prompt + completion tokens), and the peak over the first `ticks`
ticks must fit the KV pool for the run to avoid eviction.
"""
from __future__ import annotations

import argparse
import asyncio
import csv
import json
import os
import time
from collections import defaultdict, deque
from pathlib import Path

import numpy as np

from .serving import auth_headers


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
            "stream_options": {"include_usage": True}, "ignore_eos": bool(rec.get("ignore_eos", True))}
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
                chunk = json.loads(line[6:])
                if chunk.get("usage"):
                    out["prompt_tokens"] = chunk["usage"].get("prompt_tokens", 0)
                    out["cached_tokens"] = (chunk["usage"].get("prompt_tokens_details") or {}).get("cached_tokens", 0)
                if not chunk.get("choices"):
                    continue
                delta = chunk["choices"][0]
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


async def _replay(url: str, model: str, sessions: list[list[dict]], users: int,
                  duration_s: float | None = None) -> tuple[list[dict], float, int]:
    import aiohttp

    queue: asyncio.Queue = asyncio.Queue()
    for s in sessions:
        queue.put_nowait(s)
    results: list[dict] = []
    started = [0]
    timeout = aiohttp.ClientTimeout(total=None, sock_read=3600)
    async with aiohttp.ClientSession(timeout=timeout, headers=auth_headers()) as http:
        t0 = time.perf_counter()

        async def user():
            while duration_s is None or time.perf_counter() - t0 < duration_s:
                try:
                    turns = queue.get_nowait()
                except asyncio.QueueEmpty:
                    return
                started[0] += 1
                for rec in turns:  # a session's turns run in order
                    results.append(await _turn(http, url, model, rec))

        await asyncio.gather(*(user() for _ in range(max(1, users))))
        return results, time.perf_counter() - t0, started[0]


def _metric(url: str, name: str) -> float:
    import requests

    try:
        for line in requests.get(url + "/metrics", timeout=30, headers=auth_headers()).text.splitlines():
            if line.startswith(name + " "):
                return float(line.split()[1])
    except requests.RequestException:
        pass
    return 0.0


def replay(url: str, requests_path: str, users: int, model: str = "default", min_success: float = 0.99,
           duration_s: float | None = None, ttft_slo_ms: float | None = None) -> dict:
    sessions = load_sessions(requests_path)
    hits0 = _metric(url, "packmla_hicache_hit_tokens")
    prefix0 = _metric(url, "packmla_prefix_cache_hit_tokens")
    results, wall, started = asyncio.run(_replay(url, model, sessions, users, duration_s))
    ok = [r for r in results if r["ok"]]

    def pct(xs, q):
        return float(np.percentile(np.asarray(xs) * 1000, q)) if xs else None

    ttft = [r["ttft"] for r in ok if r["ttft"] is not None]
    e2e = [r["e2e"] for r in ok]
    success = len(ok) / max(1, len(results))
    expected = sum(len(s) for s in sessions[:started])
    complete = len(results) == expected
    p90 = pct(ttft, 90)
    slo_ok = ttft_slo_ms is None or (p90 is not None and p90 < ttft_slo_ms)
    return {"sessions": len(sessions), "sessions_started": started, "requests": len(results),
            "completed": len(ok), "complete": complete, "success_rate": success,
            "success_passed": success >= min_success, "ttft_slo_ms": ttft_slo_ms, "ttft_slo_passed": slo_ok,
            "passed": complete and success >= min_success and slo_ok, "users": users, "duration_s": duration_s,
            "wall_s": wall, "output_tokens": sum(r["tokens"] for r in ok),
            "output_throughput_tok_s": sum(r["tokens"] for r in ok) / wall if wall > 0 else 0.0,
            "successful_requests_per_s": len(ok) / wall if wall > 0 else 0.0,
            "ttft_ms": {"p50": pct(ttft, 50), "p90": p90, "p99": pct(ttft, 99)},
            "e2e_ms": {"p50": pct(e2e, 50), "p99": pct(e2e, 99)},
            "cache_hit_rate": (sum(r.get("cached_tokens", 0) for r in ok) / max(1, sum(r.get("prompt_tokens", 0)
                                                                                          for r in ok))),
            "hicache_restored_tokens": _metric(url, "packmla_hicache_hit_tokens") - hits0,
            "prefix_cache_hit_tokens": _metric(url, "packmla_prefix_cache_hit_tokens") - prefix0,
            "errors": [r.get("error") for r in results if not r["ok"]][:5]}


# --------------------------------------------------------------------------- request-slot FIFO
async def _request_slots(url: str, model: str, sessions: list[list[dict]], population: int, concurrency: int,
                         window_s: float, drain_s: float) -> tuple[list[dict], list[float]]:
    """`population` sessions are active at once, each with at most one ready turn; ready turns queue in
    FIFO order for `concurrency` request slots.  A finished turn puts its session's next turn at the
    tail (ready at that moment); a finished session admits the next one.  Dispatch stops at
    `window_s`; the drain waits up to `drain_s` for turns already dispatched.  Returns the finished
    turns (with ready / dispatch / completion offsets) and the ready offsets of unresolved turns."""
    import aiohttp

    origin = time.perf_counter()

    def now() -> float:
        return time.perf_counter() - origin

    pending = deque(sessions)
    ready: deque = deque()
    results: list[dict] = []

    def admit() -> None:
        if pending:
            ready.append((deque(pending.popleft()), now()))

    for _ in range(min(population, len(sessions))):
        admit()
    active: dict = {}
    timeout = aiohttp.ClientTimeout(total=None, sock_read=3600)
    async with aiohttp.ClientSession(timeout=timeout, headers=auth_headers()) as http:
        async def run_one(turns: deque, ready_s: float):
            rec = turns.popleft()
            dispatch = now()
            out = await _turn(http, url, model, rec)
            out.update(ready_s=ready_s, dispatch_s=dispatch, completed_s=dispatch + out["e2e"],
                       client_queue_ms=(dispatch - ready_s) * 1000,
                       ready_ttft_ms=None if out["ttft"] is None else (dispatch + out["ttft"] - ready_s) * 1000)
            return out, turns

        while now() < window_s and (active or ready):
            while ready and len(active) < concurrency and now() < window_s:
                turns, ready_s = ready.popleft()
                active[asyncio.ensure_future(run_one(turns, ready_s))] = ready_s
            done, _ = await asyncio.wait(list(active), timeout=max(0.0, window_s - now()),
                                         return_when=asyncio.FIRST_COMPLETED)
            for task in done:
                active.pop(task)
                out, turns = task.result()
                results.append(out)
                if turns:
                    ready.append((turns, now()))
                else:
                    admit()
        unresolved = [r for _, r in ready]
        if active:
            done, still = await asyncio.wait(list(active), timeout=drain_s)
            results.extend(task.result()[0] for task in done)
            unresolved.extend(active[task] for task in still)
            for task in still:
                task.cancel()
            await asyncio.gather(*still, return_exceptions=True)
    return results, unresolved


def slo_status(good: int, unknown: int, total: int, percentile: float = 90.0) -> str:
    """`pass` if the known-good turns alone reach the percentile, `fail` if they cannot even with every
    unknown turn good, else `indeterminate`."""
    need = percentile / 100.0 * total
    return "pass" if good >= need else ("fail" if good + unknown < need else "indeterminate")


def request_slot_replay(url: str, requests_path: str, concurrency: int, population: int, window_s: float,
                        model: str = "default", min_success: float = 0.99, ttft_slo_ms: float = 10000.0,
                        drain_s: float = 600.0) -> dict:
    """Closed-loop request-slot FIFO replay with fixed-window throughput and a ready-to-first-output SLO.

    Reference: scripts/local/business_replay/request_slots.py (`run`, `summarize`).  Throughput counts
    successful turns completed inside the window.  The SLO is the 90th percentile of the time from a
    turn becoming ready (client queue included) to its first output token, over every ready turn:
    failed or empty responses are violations, and a turn still unresolved at the end counts as a
    violation when it had already waited `ttft_slo_ms` by the cutoff, else as unknown.  The status is
    `pass` when the known-good turns alone reach 90 %, `fail` when they cannot even with every unknown
    good, and `indeterminate` otherwise."""
    if not (population >= concurrency > 0) or window_s <= 0 or drain_s <= 0:
        raise ValueError("population >= concurrency > 0 and positive window / drain required")
    sessions = load_sessions(requests_path)
    results, unresolved = asyncio.run(_request_slots(url, model, sessions, population, concurrency, window_s,
                                                     drain_s))
    ok = [r for r in results if r["ok"]]
    in_window = [r for r in ok if r["completed_s"] <= window_s]
    good = sum(1 for r in results if r["ok"] and r["ready_ttft_ms"] is not None and r["ready_ttft_ms"] < ttft_slo_ms)
    late = sum(1 for r in unresolved if (window_s - r) * 1000 >= ttft_slo_ms)
    total = len(results) + len(unresolved)
    unknown = len(unresolved) - late
    status = slo_status(good, unknown, total)

    def dist(xs):
        return {"p50": float(np.percentile(xs, 50)), "p90": float(np.percentile(xs, 90))} if xs else None

    success = len(ok) / max(1, len(results))
    return {"scheduler": "request-slot-fifo", "concurrency": concurrency, "population": population,
            "window_s": window_s, "ready_requests": total, "finished": len(results), "unresolved": len(unresolved),
            "completed": len(ok), "completed_in_window": len(in_window),
            "successful_requests_per_s": len(in_window) / window_s,
            "output_throughput_tok_s": sum(r["tokens"] for r in in_window) / window_s,
            "success_rate": success, "success_passed": success >= min_success,
            "ready_ttft_ms": dist([r["ready_ttft_ms"] for r in ok if r["ready_ttft_ms"] is not None]),
            "client_queue_ms": dist([r["client_queue_ms"] for r in results]),
            "slo": {"threshold_ms": ttft_slo_ms, "percentile": 90, "status": status, "good": good,
                    "late_unresolved": late, "unknown": unknown},
            "passed": status == "pass" and success >= min_success}


# --------------------------------------------------------------------------- sweep
def _idle_and_flush(url: str, timeout_s: float) -> None:
    """Wait until the server is healthy and idle, then flush its cache; raises RuntimeError otherwise."""
    import requests

    deadline = time.monotonic() + timeout_s
    while True:
        try:
            healthy = requests.get(url + "/health", timeout=30).status_code == 200
        except requests.RequestException:
            healthy = False
        if not healthy:
            raise RuntimeError("server unhealthy")
        if _metric(url, "packmla_num_running_reqs") == 0 and _metric(url, "packmla_num_queue_reqs") == 0:
            break
        if time.monotonic() > deadline:
            raise RuntimeError("server did not become idle")
        time.sleep(0.2)
    try:
        r = requests.post(url + "/flush_cache", timeout=60, headers=auth_headers())
    except requests.RequestException as exc:
        raise RuntimeError(f"flush failed: {exc!r}") from exc
    if r.status_code != 200:
        raise RuntimeError(f"flush failed: HTTP {r.status_code}")


_CSV_FIELDS = ("concurrency", "repeat", "passed", "complete", "success_rate", "ttft_p90_ms", "ttft_slo_passed",
               "successful_requests_per_s", "output_throughput_tok_s", "requests", "completed", "wall_s")


def sweep(url: str, requests_path: str, concurrencies: list[int], out_dir: str, *, repeats: int = 1,
          model: str = "default", duration_s: float | None = 1200.0, ttft_slo_ms: float = 10000.0,
          min_success: float = 0.99, idle_timeout_s: float = 600.0) -> dict:
    if not concurrencies or any(c <= 0 for c in concurrencies) or len(set(concurrencies)) != len(concurrencies):
        raise ValueError("concurrencies must be distinct positive integers")
    if list(concurrencies) != sorted(concurrencies):
        raise ValueError("concurrencies must be in increasing order")
    if repeats < 1 or not 0.0 <= min_success <= 1.0:
        raise ValueError("repeats >= 1 and min_success in [0, 1] required")
    root = Path(out_dir)
    root.mkdir(parents=True, exist_ok=False)  # a fresh directory per sweep
    manifest = {"base_url": url, "requests": os.path.abspath(requests_path), "concurrencies": list(concurrencies),
                "repeats": repeats, "duration_s": duration_s, "ttft_slo_ms": ttft_slo_ms,
                "min_success": min_success, "model": model}
    (root / "manifest.json").write_text(json.dumps(manifest, indent=2))
    points: list[dict] = []
    stopped = None
    for c in concurrencies:
        for rep in range(1, repeats + 1):
            try:
                _idle_and_flush(url, idle_timeout_s)
            except RuntimeError as exc:
                stopped = f"c{c} repeat {rep}: {exc}"
                break
            out = replay(url, requests_path, c, model, min_success, duration_s, ttft_slo_ms)
            d = root / f"c{c}" / f"repeat-{rep:02d}"
            d.mkdir(parents=True)
            (d / "summary.json").write_text(json.dumps(out, indent=2))
            points.append({"concurrency": c, "repeat": rep, **out})
            _write_summaries(root, points, stopped)
        if stopped:
            break
    _write_summaries(root, points, stopped)
    return {"out_dir": str(root), "points": len(points), "stopped": stopped,
            "operational_complete": stopped is None and len(points) == len(concurrencies) * repeats}


def owned_sweep(mode: str, requests_path: str, concurrencies: list[int], out_dir: str,
                startup_timeout_s: float = 1800.0, **kwargs) -> dict:
    """`sweep` against a server this call starts (packmla.server.launch with the environment's settings)
    and stops on every exit path (reference: scripts/local/sweep-lswb.sh owns one server per mode).
    The server's output goes to `<out-dir>.server.log`; the ready read-out lands in the result."""
    from ..server import launch

    env = dict(os.environ)
    cmd, extra = launch.resolve(mode, env)
    env.update(extra)
    group = launch.ServerGroup(cmd, env, f"{out_dir.rstrip('/')}.server.log")
    url = f"http://127.0.0.1:{env.get('PORT', '30000')}"
    try:
        info = launch.wait_ready(url, group, startup_timeout_s)
        out = sweep(url, requests_path, concurrencies, out_dir, **kwargs)
        out["server"] = {"mode": mode, "command": cmd,
                         **{k: info.get(k) for k in ("kv_cache_format", "max_total_num_tokens", "prefix_cache")}}
        return out
    finally:
        group.stop()


def _write_summaries(root: Path, points: list[dict], stopped: str | None) -> None:
    (root / "summary.json").write_text(json.dumps({"points": points, "stopped": stopped}, indent=2))
    with open(root / "summary.csv", "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=_CSV_FIELDS)
        w.writeheader()
        for p in points:
            w.writerow({k: (p["ttft_ms"]["p90"] if k == "ttft_p90_ms" else p.get(k)) for k in _CSV_FIELDS})


# --------------------------------------------------------------------------- capacity plan
def request_tokens(rec: dict) -> int:
    """Prompt + completion tokens of one recorded request: the record's own counts when present
    (`prompt_tokens`), else the UTF-8 bytes of its message contents (the byte tokenizer's count)."""
    prompt = rec.get("prompt_tokens")
    if prompt is None:
        prompt = sum(len(str(m.get("content", "")).encode()) for m in rec["messages"])
    return int(prompt) + int(rec.get("max_tokens", 256))


def peak_live_tokens(sessions: list[list[dict]], concurrency: int, ticks: int | None = None) -> int:
    """Largest sum of the active requests' sizes over the first `ticks` ticks of C session slots."""
    pending = deque([request_tokens(r) for r in s] for s in sessions)
    slots: list[deque] = []
    peak = tick = 0
    while (pending or slots) and (ticks is None or tick < ticks):
        while len(slots) < concurrency and pending:
            slots.append(deque(pending.popleft()))
        peak = max(peak, sum(s[0] for s in slots))
        for s in slots:
            s.popleft()
        slots = [s for s in slots if s]
        tick += 1
    return peak


def plan(requests_path: str, concurrencies: list[int], pool_tokens: int, ticks: int | None = None) -> dict:
    sessions = load_sessions(requests_path)
    rows = [{"concurrency": c, "peak_live_tokens": peak_live_tokens(sessions, c, ticks)} for c in concurrencies]
    for r in rows:
        r["utilization"] = r["peak_live_tokens"] / pool_tokens
        r["fits"] = r["peak_live_tokens"] <= pool_tokens
    fitting = [r["concurrency"] for r in rows if r["fits"]]
    return {"pool_tokens": pool_tokens, "ticks": ticks, "points": rows,
            "largest_fitting_concurrency": max(fitting) if fitting else None}


def _ints(text: str) -> list[int]:
    return [int(x) for x in text.split(",") if x.strip()]


def main(argv=None) -> dict:
    import sys

    argv = list(sys.argv[1:] if argv is None else argv)
    cmd = argv.pop(0) if argv and argv[0] in ("sweep", "plan") else "replay"
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--requests", required=True)
    if cmd == "plan":
        ap.add_argument("--concurrencies", type=_ints, required=True)
        ap.add_argument("--pool-tokens", type=int, required=True)
        ap.add_argument("--ticks", type=int, default=None)
        a = ap.parse_args(argv)
        out = plan(a.requests, a.concurrencies, a.pool_tokens, a.ticks)
        print(json.dumps(out, indent=2))
        return out
    ap.add_argument("--base-url", default="http://127.0.0.1:30000")
    ap.add_argument("--model", default="default")
    ap.add_argument("--min-success", type=float, default=0.99)
    ap.add_argument("--duration-s", type=float, default=None)
    ap.add_argument("--ttft-slo-ms", type=float, default=None)
    if cmd == "sweep":
        ap.add_argument("--concurrencies", type=_ints, required=True)
        ap.add_argument("--repeats", type=int, default=1)
        ap.add_argument("--out-dir", required=True)
        ap.add_argument("--launch", choices=["native", "direct"], default=None,
                        help="own one server of this mode for the sweep (packmla.server.launch, its environment "
                             "names), stopped on every exit path; --base-url is then derived from PORT")
        ap.add_argument("--startup-timeout", type=float, default=1800.0)
        a = ap.parse_args(argv)
        kwargs = dict(repeats=a.repeats, model=a.model,
                      duration_s=a.duration_s if a.duration_s is not None else 1200.0,
                      ttft_slo_ms=a.ttft_slo_ms if a.ttft_slo_ms is not None else 10000.0, min_success=a.min_success)
        if a.launch:
            out = owned_sweep(a.launch, a.requests, a.concurrencies, a.out_dir, a.startup_timeout, **kwargs)
        else:
            out = sweep(a.base_url, a.requests, a.concurrencies, a.out_dir, **kwargs)
        print(json.dumps(out, indent=2))
        if not out["operational_complete"]:
            raise SystemExit(f"sweep stopped: {out['stopped']}")
        return out
    ap.add_argument("--users", type=int, default=24, help="active users (session) or request slots (request-slot)")
    ap.add_argument("--scheduler", choices=["session", "request-slot"], default="session")
    ap.add_argument("--population", type=int, default=None, help="request-slot: active sessions (default: --users)")
    ap.add_argument("--drain-s", type=float, default=600.0)
    ap.add_argument("--output", default=None)
    a = ap.parse_args(argv)
    if a.scheduler == "request-slot":
        if a.duration_s is None:
            ap.error("--scheduler request-slot needs --duration-s (the fixed measurement window)")
        out = request_slot_replay(a.base_url, a.requests, a.users, a.population or a.users, a.duration_s, a.model,
                                  a.min_success, a.ttft_slo_ms if a.ttft_slo_ms is not None else 10000.0, a.drain_s)
        print(json.dumps(out, indent=2))
        if not out["passed"]:
            raise SystemExit(f"replay gates failed: slo={out['slo']['status']} success={out['success_rate']:.4f}")
        return out
    out = replay(a.base_url, a.requests, a.users, a.model, a.min_success, a.duration_s, a.ttft_slo_ms)
    text = json.dumps(out, indent=2)
    if a.output:
        with open(a.output, "x") as f:
            f.write(text)
    print(text)
    if not out["passed"]:
        raise SystemExit(f"replay gates failed: complete={out['complete']} success={out['success_rate']:.4f} "
                         f"ttft_p90_ms={out['ttft_ms']['p90']}")
    return out


if __name__ == "__main__":
    main()

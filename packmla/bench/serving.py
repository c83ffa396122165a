"""Serving benchmark client for an OpenAI-compatible server (packmla's or any other).

    python -m packmla.bench.serving --base-url http://127.0.0.1:30000 --dataset random \
        --input-len 32768 --output-len 256 --concurrency 8 [--flush-cache]
    python -m packmla.bench.serving ... --dataset shared-prefix --prefix-len 4096 --num-groups 4
    python -m packmla.bench.serving ... --dataset multi-turn --turns 4 --sessions 8

Protocol of the reference's random-text client (scripts/local/bench-serving.sh:64-111, :153-192):
a warm-up phase of C requests, then a measured phase of 3C requests at concurrency C, the cache
flushed before each phase (`/flush_cache`), every request forced to exactly `output-len` tokens
(`ignore_eos`), and the output length of every response validated.  Token-id prompts avoid any
tokenizer dependence.  Metrics: output tokens/s, request throughput, TTFT / TPOT / E2E latency
(mean, p50, p99) from streamed responses.
The multi-turn dataset re-sends each session's growing history every turn (the workload that the
HiCache host tier serves).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Result:
    ok: bool
    prompt_len: int
    output_ids: list[int] = field(default_factory=list)
    ttft: float = 0.0
    e2e: float = 0.0
    itl: list[float] = field(default_factory=list)
    error: str = ""


def random_prompts(n: int, input_len: int, vocab: int, seed: int) -> list[list[int]]:
    rng = random.Random(seed)
    return [[rng.randrange(3, vocab) for _ in range(input_len)] for _ in range(n)]


def shared_prefix_prompts(n: int, prefix_len: int, suffix_len: int, groups: int, vocab: int, seed: int):
    rng = random.Random(seed)
    prefixes = [[rng.randrange(3, vocab) for _ in range(prefix_len)] for _ in range(groups)]
    return [prefixes[i % groups] + [rng.randrange(3, vocab) for _ in range(suffix_len)] for i in range(n)]


async def _request(session, url: str, model: str, prompt: list[int], output_len: int) -> Result:
    body = {"model": model, "prompt": prompt, "max_tokens": output_len, "temperature": 0.0, "stream": True,
            "ignore_eos": True}
    res = Result(False, len(prompt))
    t0 = time.perf_counter()
    last = t0
    try:
        async with session.post(url + "/v1/completions", json=body) as resp:
            if resp.status != 200:
                res.error = f"HTTP {resp.status}: {await resp.text()}"
                return res
            async for raw in resp.content:
                line = raw.decode().strip()
                if not line.startswith("data: ") or line == "data: [DONE]":
                    continue
                chunk = json.loads(line[6:])
                ids = chunk["choices"][0].get("token_ids") or []
                if ids:
                    now = time.perf_counter()
                    if not res.output_ids:
                        res.ttft = now - t0
                    else:
                        res.itl.append(now - last)
                    last = now
                    res.output_ids.extend(ids)
        res.e2e = time.perf_counter() - t0
        res.ok = len(res.output_ids) == output_len
        if not res.ok:
            res.error = f"expected {output_len} tokens, got {len(res.output_ids)}"
    except Exception as exc:  # network errors count as failed requests
        res.error = repr(exc)
    return res


async def run_phase(url: str, model: str, prompts: list[list[int]], output_len: int, concurrency: int):
    import aiohttp

    sem = asyncio.Semaphore(concurrency)
    timeout = aiohttp.ClientTimeout(total=None, sock_read=3600)
    async with aiohttp.ClientSession(timeout=timeout, headers=auth_headers()) as session:
        async def one(p):
            async with sem:
                return await _request(session, url, model, p, output_len)

        t0 = time.perf_counter()
        results = await asyncio.gather(*(one(p) for p in prompts))
        return results, time.perf_counter() - t0


def summarize(results: list[Result], wall: float) -> dict:
    ok = [r for r in results if r.ok]
    out_tokens = sum(len(r.output_ids) for r in ok)

    def stats(xs):
        if not xs:
            return {"mean": None, "p50": None, "p99": None}
        a = np.asarray(xs) * 1000
        return {"mean": float(a.mean()), "p50": float(np.percentile(a, 50)), "p99": float(np.percentile(a, 99))}

    tpot = [(r.e2e - r.ttft) / max(1, len(r.output_ids) - 1) for r in ok]
    return {"requests": len(results), "completed": len(ok), "success_rate": len(ok) / max(1, len(results)),
            "wall_s": wall, "output_throughput_tok_s": out_tokens / wall if wall > 0 else 0.0,
            "request_throughput": len(ok) / wall if wall > 0 else 0.0,
            "total_input_tokens": sum(r.prompt_len for r in ok), "total_output_tokens": out_tokens,
            "ttft_ms": stats([r.ttft for r in ok]), "tpot_ms": stats(tpot), "e2e_ms": stats([r.e2e for r in ok]),
            "output_lens": [len(r.output_ids) for r in results],
            "validated": len(ok) == len(results) > 0,  # every request completed with exactly output-len tokens
            "errors": [r.error for r in results if not r.ok][:5]}


def phase_summaries(out: dict) -> list[tuple[str, dict]]:
    """(name, summary) of every measured wave of a `bench` result."""
    if "turns" in out:
        return [(f"turn{i}", t) for i, t in enumerate(out["turns"])]
    return [(k, out[k]) for k in ("warmup", "measured") if k in out]


def write_records(path: str, out: dict) -> None:
    """One JSON line per wave (reference: bench-serving.sh writes and validates one record per wave);
    the file must not exist."""
    with open(path, "x") as f:
        for name, summary in phase_summaries(out):
            f.write(json.dumps({"phase": name, "dataset": out["dataset"], "concurrency": out["concurrency"],
                                "input_len": out["input_len"], "output_len": out["output_len"], **summary}) + "\n")


def auth_headers() -> dict:
    """`Authorization: Bearer ...` from PACKMLA_API_KEY (or OPENAI_API_KEY) for a server started with
    --api-key; empty otherwise."""
    import os

    key = os.environ.get("PACKMLA_API_KEY") or os.environ.get("OPENAI_API_KEY")
    return {"Authorization": f"Bearer {key}"} if key else {}


def flush(url: str) -> None:
    import requests

    requests.post(url + "/flush_cache", timeout=60, headers=auth_headers()).raise_for_status()


def server_info(url: str) -> dict:
    import requests

    return requests.get(url + "/server_info", timeout=60, headers=auth_headers()).json()


def resolve_concurrency(requested, info: dict, input_len: int, output_len: int) -> int:
    """`auto`: as many complete requests as the running server's KV pool holds (reference:
    scripts/local/bench-serving.sh `auto`); rejects a request that exceeds the server's context."""
    ctx = info.get("context_length")
    if ctx is not None and input_len + output_len > ctx:
        raise SystemExit(f"input + output = {input_len + output_len} exceeds the server's context {ctx}")
    if requested == "auto":
        c = int(info["max_total_num_tokens"]) // (input_len + output_len)
        if c < 1:
            raise SystemExit("the server's KV pool cannot hold one complete request")
        return c
    c = int(requested)
    if c < 1:
        raise SystemExit("concurrency must be a positive integer or auto")
    return c


def bench(url: str, dataset: str, input_len: int, output_len: int, concurrency: int | str, *, vocab: int | None = None,
          model: str = "default", flush_cache: bool = True, seed: int = 0, prefix_len: int = 0, num_groups: int = 1,
          turns: int = 1, sessions: int = 0) -> dict:
    info = server_info(url)
    concurrency = resolve_concurrency(concurrency, info, input_len, output_len)
    vocab = vocab or info.get("model_config", {}).get("vocab_size", 32000)
    n_warm, n_meas = concurrency, 3 * concurrency
    out = {"dataset": dataset, "concurrency": concurrency, "input_len": input_len, "output_len": output_len,
           "server": {k: info.get(k) for k in ("kv_cache_format", "max_total_num_tokens", "tp",
                                               "enable_hierarchical_cache")}}
    if dataset == "multi-turn":
        rng = random.Random(seed)
        hist = [[rng.randrange(3, vocab) for _ in range(input_len)] for _ in range(sessions or concurrency)]
        phases = []
        for t in range(turns):
            if flush_cache and t == 0:
                flush(url)
            res, wall = asyncio.run(run_phase(url, model, hist, output_len, concurrency))
            phases.append(summarize(res, wall))
            hist = [h + r.output_ids + [rng.randrange(3, vocab) for _ in range(64)] for h, r in zip(hist, res)]
        out["turns"] = phases
        return out
    if dataset == "random":
        prompts = random_prompts(n_warm + n_meas, input_len, vocab, seed)
    elif dataset == "shared-prefix":
        prompts = shared_prefix_prompts(n_warm + n_meas, prefix_len, input_len, num_groups, vocab, seed)
    else:
        raise ValueError(f"unknown dataset {dataset}")
    for name, batch in (("warmup", prompts[:n_warm]), ("measured", prompts[n_warm:])):
        if flush_cache:
            flush(url)
        res, wall = asyncio.run(run_phase(url, model, batch, output_len, concurrency))
        out[name] = summarize(res, wall)
    return out


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--base-url", default="http://127.0.0.1:30000")
    ap.add_argument("--model", default="default")
    ap.add_argument("--dataset", choices=["random", "shared-prefix", "multi-turn"], default="random")
    ap.add_argument("--input-len", type=int, default=32768)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--concurrency", default="8", help="a positive integer, or auto (what the KV pool holds)")
    ap.add_argument("--prefix-len", type=int, default=0)
    ap.add_argument("--num-groups", type=int, default=1)
    ap.add_argument("--turns", type=int, default=4)
    ap.add_argument("--sessions", type=int, default=0)
    ap.add_argument("--flush-cache", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--output-file", default=None, help="write one JSON record per wave here (a new file)")
    a = ap.parse_args(argv)
    out = bench(a.base_url, a.dataset, a.input_len, a.output_len, a.concurrency, model=a.model,
                flush_cache=a.flush_cache, seed=a.seed, prefix_len=a.prefix_len, num_groups=a.num_groups,
                turns=a.turns, sessions=a.sessions)
    print(json.dumps(out, indent=2))
    if a.output_file:
        write_records(a.output_file, out)
    bad = [name for name, summary in phase_summaries(out) if not summary["validated"]]
    if bad:  # incomplete requests, wrong output lengths or request errors fail the run
        raise SystemExit(f"waves failed validation: {', '.join(bad)}")
    return out


if __name__ == "__main__":
    main()

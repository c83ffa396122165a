"""Serving runner: checkpoint check, server launch, smoke, serving benchmark, stop, sealed record.

    TP=4 MODEL=v4-flash python -m packmla.bench.serve_runner RUN_DIR direct \
        [--checkpoint DIR --profile dsv4] [--input-len 32768 --output-len 256 --concurrency 8] [--smoke-only]

Reference behaviour: scripts/modal/serve.py (`download_model` and checkpoint inspection,
`_running_serving_server`, `benchmark_serving`, the model smokes).  There is no network here, so a
checkpoint is verified against its pinned profile (packmla.utils.model_profiles) instead of downloaded.
Steps, each recorded in `RUN_DIR/steps.json`:

  1. checkpoint: with --checkpoint, the directory must match the pinned profile (config sha256, shards);
  2. launch: the server starts through packmla.server.launch's process-group owner, with the launcher's
     environment settings (TP, PORT, MEM_FRAC, ...); the pool read out of /server_info is recorded;
  3. smoke: a few completions of random token prompts must return exactly max_tokens tokens
     (EOS ignored), and /metrics must answer;
  4. benchmark: packmla.bench.serving's random-text protocol (C warm-up + 3C measured, cache flushed)
     unless --smoke-only; every wave must validate;
  5. stop: the server's process group is stopped on every path (success, failure, interrupt).

The run directory is then sealed (manifest.json + SHA256SUMS).  Exit code 0 only if every step passed.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
import time
from pathlib import Path


def smoke(url: str, vocab: int, n: int = 3, max_tokens: int = 8, prompt_len: int = 64) -> dict:
    import requests

    from .serving import auth_headers

    rng = random.Random(0)
    results = []
    for i in range(n):
        prompt = [rng.randrange(3, vocab) for _ in range(prompt_len)]
        r = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": max_tokens,
                                                         "temperature": 0.0, "ignore_eos": True},
                          headers=auth_headers(), timeout=600)
        ok = r.status_code == 200 and len(r.json()["choices"][0]["token_ids"]) == max_tokens
        results.append({"request": i, "status": r.status_code, "ok": ok})
    metrics = requests.get(url + "/metrics", timeout=30, headers=auth_headers())
    return {"passed": all(x["ok"] for x in results) and metrics.status_code == 200, "requests": results}


def run(run_dir: Path, mode: str, env: dict, *, checkpoint: Path | None = None, profile: str | None = None,
        input_len: int = 32768, output_len: int = 256, concurrency: int | str = 8, smoke_only: bool = False,
        wait_timeout: float = 1800.0, seal: bool = True) -> dict:
    from ..server.launch import ServerGroup, resolve, wait_ready
    from ..utils.model_profiles import verify_checkpoint

    run_dir = Path(run_dir)
    if run_dir.exists() and any(run_dir.iterdir()):
        raise ValueError(f"fresh run directory required: {run_dir}")
    run_dir.mkdir(parents=True, exist_ok=True)
    steps: list[dict] = []

    def record(name, ok, **kw):
        steps.append({"step": name, "passed": bool(ok), **kw})
        (run_dir / "steps.json").write_text(json.dumps(steps, indent=1) + "\n")
        return ok

    ok = True
    if checkpoint is not None:
        try:
            ok = record("checkpoint", True, **verify_checkpoint(profile, checkpoint))
        except ValueError as exc:
            ok = record("checkpoint", False, error=str(exc))
    group = None
    url = f"http://127.0.0.1:{env.get('PORT', '30000')}"
    try:
        if ok:
            cmd, extra = resolve(mode, env)
            group = ServerGroup(cmd, {**os.environ, **extra}, log_path=str(run_dir / "server.log"))
            t0 = time.time()
            try:
                info = wait_ready(url, group, wait_timeout)
                ok = record("launch", True, seconds=round(time.time() - t0, 1), command=cmd,
                            pool={k: info.get(k) for k in ("kv_cache_format", "max_total_num_tokens", "tp",
                                                           "num_pages", "max_running_requests")})
            except RuntimeError as exc:
                info = {}
                ok = record("launch", False, error=str(exc), command=cmd)
        if ok:
            vocab = info.get("model_config", {}).get("vocab_size") or 32000
            s = smoke(url, vocab)
            ok = record("smoke", s["passed"], **s)
        if ok and not smoke_only:
            from .serving import bench, phase_summaries

            out = bench(url, "random", input_len, output_len, concurrency, flush_cache=True)
            (run_dir / "serving.json").write_text(json.dumps(out, indent=1) + "\n")
            bad = [name for name, summary in phase_summaries(out) if not summary["validated"]]
            ok = record("benchmark", not bad, failed_waves=bad,
                        measured=out.get("measured", {}).get("output_throughput_tok_s"))
    finally:
        if group is not None:
            rc = group.stop()
            record("stop", True, exit_code=rc)
    passed = all(s["passed"] for s in steps) and any(s["step"] == "smoke" for s in steps)
    if seal:
        from ..utils.provenance import seal_run

        seal_run(run_dir, command=[sys.executable, "-m", "packmla.bench.serve_runner"] + sys.argv[1:],
                 extra={"mode": mode, "passed": passed,
                        "settings": {k: env[k] for k in ("MODEL", "TP", "PORT", "DEVICE", "MEM_FRAC") if k in env}})
    return {"run_dir": str(run_dir), "passed": passed, "steps": steps}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("run_dir", type=Path)
    ap.add_argument("mode", choices=["native", "direct"])
    ap.add_argument("--checkpoint", type=Path, default=None)
    ap.add_argument("--profile", default="dsv4")
    ap.add_argument("--input-len", type=int, default=32768)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--concurrency", default="8")
    ap.add_argument("--smoke-only", action="store_true")
    ap.add_argument("--wait-timeout", type=float, default=1800.0)
    a = ap.parse_args(argv)
    conc = a.concurrency if a.concurrency == "auto" else int(a.concurrency)
    out = run(a.run_dir, a.mode, dict(os.environ), checkpoint=a.checkpoint, profile=a.profile,
              input_len=a.input_len, output_len=a.output_len, concurrency=conc, smoke_only=a.smoke_only,
              wait_timeout=a.wait_timeout)
    print(json.dumps({"run_dir": out["run_dir"], "passed": out["passed"]}))
    return 0 if out["passed"] else 1


if __name__ == "__main__":
    sys.exit(main())

"""Shared-prefix serving workload through the engine, prefix cache on and off.

    python -m packmla.bench.shared_prefix --groups 4 --prompts-per-group 8 --system-len 16384 \
        --question-len 512 --output-len 64 --concurrency 8 [--modes on,off]

Reference workload: SGLang's generated-shared-prefix dataset as the reference runs it
(benchmarks/serving/shared-prefix-g32-c16-n3-20261020/README.md: 32 groups x 40 prompts, a 128k system
prompt + 512-token question, 256 output tokens, concurrency 16).  Here the same shape, scaled by the flags,
runs in process through `Engine.step()` on the V4-Flash-shape model (random init, Direct KV): all prompts
are submitted at once in group-interleaved order and the engine keeps at most `concurrency` running.  Per
mode it reports requests/s and output tokens/s over the wall time, the mean and p90 time to first token
from submission, and how many prompt tokens were prefilled versus taken from shared prefix blocks.
"""
from __future__ import annotations

import argparse
import json
import random
import time


def prompts(groups: int, per_group: int, system_len: int, question_len: int, vocab: int, seed: int):
    rng = random.Random(seed)
    systems = [[rng.randrange(3, vocab) for _ in range(system_len)] for _ in range(groups)]
    return [systems[i % groups] + [rng.randrange(3, vocab) for _ in range(question_len)]
            for i in range(groups * per_group)]


def run(eng, plist, output_len: int, device) -> dict:
    import torch

    from ..engine.engine import SamplingParams

    params = SamplingParams(max_new_tokens=output_len, temperature=0.0, ignore_eos=True)
    before = eng.metrics.snapshot()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    rids = [eng.add_request(p, params) for p in plist]
    while eng.has_work():
        eng.step()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    wall = time.perf_counter() - t0
    m = eng.metrics.snapshot()
    reqs = [eng.result(r) for r in rids]
    ttft = sorted(r.t_first_token - t0 for r in reqs)
    out_tokens = sum(len(r.output_ids) for r in reqs)
    prefill = m.get("prefill_tokens", 0) - before.get("prefill_tokens", 0)
    hits = m.get("prefix_block_hit_tokens", 0) - before.get("prefix_block_hit_tokens", 0)
    total_prompt = sum(len(p) for p in plist)
    return {"requests": len(plist), "wall_s": round(wall, 3), "requests_per_s": round(len(plist) / wall, 4),
            "output_tokens_per_s": round(out_tokens / wall, 2), "ttft_mean_s": round(sum(ttft) / len(ttft), 3),
            "ttft_p90_s": round(ttft[int(0.9 * (len(ttft) - 1))], 3), "prompt_tokens": total_prompt,
            "prefilled_tokens": prefill, "block_hit_tokens": hits,
            "device_hit_fraction": round(1 - prefill / total_prompt, 4)}


def main(argv=None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--groups", type=int, default=4)
    ap.add_argument("--prompts-per-group", type=int, default=8)
    ap.add_argument("--system-len", type=int, default=16384)
    ap.add_argument("--question-len", type=int, default=512)
    ap.add_argument("--output-len", type=int, default=64)
    ap.add_argument("--concurrency", type=int, default=8)
    ap.add_argument("--modes", default="on,off", help="prefix cache settings to run, in order")
    ap.add_argument("--seed", type=int, default=42)
    args = ap.parse_args(argv)

    import torch

    from ..config import ModelConfig
    from ..parallel.comm import TPComm
    from .engine_setup import build_engine
    from .timing import ClockSampler

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = ModelConfig()
    plist = prompts(args.groups, args.prompts_per_group, args.system_len, args.question_len, cfg.vocab_size,
                    args.seed)
    rows = []
    for mode in args.modes.split(","):
        eng, _ = build_engine(cfg, device, 0, 1, TPComm(), args.concurrency, args.system_len + args.question_len,
                              args.output_len, "direct", prefix_cache=(mode == "on"))
        eng.runner.capture()
        with ClockSampler(0) as clk:
            row = run(eng, plist, args.output_len, device)
        row.update(mode=f"prefix cache {mode}", groups=args.groups, prompts_per_group=args.prompts_per_group,
                   system_len=args.system_len, question_len=args.question_len, output_len=args.output_len,
                   concurrency=args.concurrency, clocks=clk.summary())
        print(json.dumps(row), flush=True)
        rows.append(row)
        eng.runner.release()
        del eng
        torch.cuda.empty_cache()
    return rows


if __name__ == "__main__":
    main()

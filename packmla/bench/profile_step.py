"""Kernel-time breakdown of one decode step (diagnostics; numbers taken under a profiler are not
benchmark values).

    python -m packmla.bench.profile_step --concurrency 40 --context 32768 --out profile.txt
"""
from __future__ import annotations

import argparse
import time

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--concurrency", type=int, default=40)
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--kv-format", default="direct")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--out", default=None)
    ap.add_argument("--rows", type=int, default=40)
    args = ap.parse_args()

    from packmla.bench.synthetic import fill_synthetic
    from packmla.config import EngineConfig, ModelConfig
    from packmla.engine.engine import Engine
    from packmla.kv.pool import bytes_per_full_token, fixed_bytes

    dev = torch.device("cuda", 0)
    cfg = ModelConfig()
    C = args.concurrency
    max_context = args.context + 512
    ecfg = EngineConfig(kv_cache_format=args.kv_format, max_running_requests=C, cuda_graph_bs=[C])
    bpt = bytes_per_full_token(cfg, args.kv_format, ecfg.swa_full_tokens_ratio)
    kv_bytes = int((C * (max_context // 256 + 1) + 8) * 256 * bpt) + fixed_bytes(cfg, C + 1) + (64 << 20)
    eng = Engine.build(cfg, ecfg, dev, max_context=max_context, max_requests=C, kv_bytes=kv_bytes)
    fill_synthetic(eng, C, args.context, 64)
    m = eng.model
    tokens = torch.tensor([r.output_ids[-1] for r in eng.running], device=dev)
    pos = torch.tensor([r.context_len - 1 for r in eng.running], device=dev)
    slots = torch.tensor([r.slot for r in eng.running], device=dev)
    m.decode(tokens, pos, slots)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    m.decode(tokens, pos + 1, slots)
    torch.cuda.synchronize(dev)
    eager_ms = (time.perf_counter() - t0) * 1e3
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        for s in range(args.steps):
            m.decode(tokens, pos + 2 + s, slots)
        torch.cuda.synchronize(dev)
    table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=args.rows)
    text = f"eager step wall ms: {eager_ms:.2f}  (steps profiled: {args.steps})\n{table}\n"
    print(text)
    if args.out:
        with open(args.out, "w") as f:
            f.write(text)


if __name__ == "__main__":
    main()

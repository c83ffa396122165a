"""Measured KV-pool capacity, Native vs Packed, on one GPU at a memory fraction.

    python -m packmla.bench.capacity [--tp 4] [--mem-fraction-static 0.88] [--max-running-requests 256]

The reference's headline capacity figure is the pool each TP4 rank allocated at `--mem-fraction-static 0.88`
with the model loaded: 3,745,536 Native and 4,536,832 Packed token slots, 1.2113x (docs/report.md:30).  This
tool reproduces that measurement on one GPU: it loads the weight shard of rank 0 of a TP=`--tp` deployment of
the V4-Flash-shape model (random init; every rank holds the full latent KV of every token, so one rank's pool
is the deployment's token capacity), sizes the pool the way the serving engine does (memory fraction x total
device memory - the resident weights and per-request state), allocates it for real in each format and prints
the token slots of both and their ratio.
"""
from __future__ import annotations

import argparse
import json
import time


def measure(tp: int, mem_fraction: float, max_running: int, device=None) -> dict:
    import torch

    from ..config import EngineConfig, ModelConfig
    from ..kv.pool import KVPool, plan_capacity
    from ..models.weights import init_weights
    from ..ops.moe import prepare_experts_mx

    dev = torch.device(device or "cuda")
    cfg = ModelConfig()
    torch.cuda.synchronize(dev)
    t0 = time.time()
    W = init_weights(cfg, 0, tp, dev, seed=0)
    for lw in W["layers"]:
        prepare_experts_mx(lw, drop_canonical=True)
    torch.cuda.synchronize(dev)
    total = torch.cuda.get_device_properties(dev).total_memory
    weights = torch.cuda.memory_allocated(dev)
    budget = int(total * mem_fraction) - weights
    out = {"tp": tp, "mem_fraction_static": mem_fraction, "total_gib": round(total / 2 ** 30, 2),
           "weights_gib": round(weights / 2 ** 30, 2), "kv_budget_gib": round(budget / 2 ** 30, 2),
           "load_s": round(time.time() - t0, 1)}
    for fmt in ("native", "direct"):
        ecfg = EngineConfig(kv_cache_format=fmt, tp=tp, max_running_requests=max_running,
                            mem_fraction_static=mem_fraction)
        cap = plan_capacity(cfg, ecfg, budget)
        pool = KVPool(cfg, ecfg, cap.num_pages, max_running + 1, 1 << 20, dev)  # allocated: it must fit
        torch.cuda.synchronize(dev)
        out[fmt] = {"token_slots": cap.max_total_tokens, "pages": cap.num_pages,
                    "bytes_per_token": round(cap.bytes_per_full_token, 2),
                    "pool_gib": round((torch.cuda.memory_allocated(dev) - weights) / 2 ** 30, 2)}
        del pool
        torch.cuda.empty_cache()
    out["packed_vs_native"] = round(out["direct"]["token_slots"] / out["native"]["token_slots"], 4)
    out["reference"] = {"native": 3745536, "packed": 4536832, "ratio": 1.2113, "hardware": "4xH100 80GB TP4"}
    return out


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--tp", type=int, default=4, help="tensor-parallel size whose rank-0 weight shard is loaded")
    ap.add_argument("--mem-fraction-static", type=float, default=0.88)
    ap.add_argument("--max-running-requests", type=int, default=256)
    args = ap.parse_args(argv)
    res = measure(args.tp, args.mem_fraction_static, args.max_running_requests)
    print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()

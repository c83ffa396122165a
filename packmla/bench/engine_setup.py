"""Engine construction shared by the serving benchmark (`bench.py`) and the step breakdown
(`python -m packmla.bench.step_breakdown`): the V4-Flash-shape model, a pool sized for C requests of
`prompt_len + output_len` tokens, CUDA-graph buckets up to C, TP = EP = world."""
from __future__ import annotations

import math

DEFAULT_CONCURRENCY = {1: 8, 2: 8, 4: 24, 8: 40}


def graph_buckets(concurrency: int) -> list[int]:
    return [b for b in (1, 2, 4, 8, 16, 24, 32, 40, 48, 64) if b < concurrency] + [concurrency]


def build_engine(cfg, device, rank: int, world: int, comm, concurrency: int, prompt_len: int, output_len: int,
                 kv_format: str = "direct", seed: int = 0, dp_attention: bool = False, prefix_cache: bool = True):
    """-> (engine, max_context).  The pool holds every request's pages plus a few spare pages; with DP
    attention each rank serves concurrency / world requests, so its pool and graph buckets are sized for
    those."""
    from ..config import EngineConfig
    from ..engine.engine import Engine
    from ..kv.pool import bytes_per_full_token, fixed_bytes

    C = concurrency // world if dp_attention else concurrency
    max_context = prompt_len + output_len + 256
    ecfg = EngineConfig(kv_cache_format=kv_format, tp=world, ep=world, max_running_requests=C,
                        cuda_graph_bs=graph_buckets(C), chunked_prefill_size=8192, prefix_cache=prefix_cache,
                        dp_attention=dp_attention)
    pages_per_req = math.ceil(max_context / 256)
    bpt = bytes_per_full_token(cfg, kv_format, ecfg.swa_full_tokens_ratio)
    kv_bytes = int((C * pages_per_req + 8) * 256 * bpt) + fixed_bytes(cfg, C + 1) + (64 << 20)
    eng = Engine.build(cfg, ecfg, device, rank, world, comm, max_context=max_context, max_requests=C,
                       kv_bytes=kv_bytes, seed=seed)
    return eng, max_context

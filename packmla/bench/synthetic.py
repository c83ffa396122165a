"""Synthetic serving state: requests whose KV cache holds `context` tokens of random latents.

Used by the decode benchmark so a 32k-token context per request does not need a full prefill:
every C4 / C128 record and every SWA ring row is written by the same store kernels the engine
uses (random-normal raw latents), index keys are random FP8, and the request is placed in the
running set with `context` prompt tokens.  The decode steps that follow read exactly the bytes a
real prefill would have produced in shape and layout.
"""
from __future__ import annotations

import torch

from ..engine.engine import Engine, Request, SamplingParams
from ..formats import abi
from ..ops import indexer as idx_ops
from ..ops import kv as kv_ops


def fill_synthetic(engine: Engine, n_requests: int, context: int, max_new_tokens: int, seed: int = 0,
                   chunk_rows: int = 1 << 16) -> list[Request]:
    pool, model, cfg = engine.pool, engine.model, engine.cfg
    dev = pool.device
    if context % abi.C128_RATIO:
        raise ValueError("synthetic context must be a multiple of 128")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    reqs = []
    for i in range(n_requests):
        slot = pool.admit(context + max_new_tokens + 1)
        req = Request(rid=next(engine._ids), prompt=[0] * context,
                      params=SamplingParams(max_new_tokens=max_new_tokens), slot=slot, prefilled=context)
        req.output_ids.append(int(torch.randint(0, cfg.vocab_size, (1,), generator=gen, device=dev)))
        reqs.append(req)
    slots = torch.tensor([r.slot for r in reqs], device=dev, dtype=torch.int64)
    n4 = context // abi.C4_RATIO
    n128 = context // abi.C128_RATIO
    r4 = torch.arange(n4, device=dev)
    pt = pool.page_table[slots].long()
    phys4 = (pt[:, r4 // abi.RECORDS_PER_PAGE] * abi.RECORDS_PER_PAGE + r4 % abi.RECORDS_PER_PAGE).reshape(-1)
    pos4 = (r4 * abi.C4_RATIO).repeat(n_requests)
    r2 = torch.arange(n128, device=dev)
    ct = pool.c128_table[slots].long()
    phys2 = (ct[:, r2 // abi.RECORDS_PER_PAGE] * abi.RECORDS_PER_PAGE + r2 % abi.RECORDS_PER_PAGE).reshape(-1)
    pos2 = (r2 * abi.C128_RATIO).repeat(n_requests)
    w = cfg.window
    ring = (slots[:, None] * w + torch.arange(w, device=dev)[None]).reshape(-1)
    ring_pos = (context - w + torch.arange(w, device=dev)).repeat(n_requests)  # ring index == pos % w
    eps = cfg.rms_eps

    def rand_rows(n):
        t = torch.empty(n, abi.LATENT_DIM, device=dev, dtype=torch.float32)
        return t.normal_(generator=gen)

    for layer in range(cfg.num_layers):
        lw = model.W["layers"][layer]
        for a in range(0, ring.numel(), chunk_rows):
            b = min(ring.numel(), a + chunk_rows)
            kv_ops.native_store(rand_rows(b - a), lw["kv_norm"], eps, ring[a:b], ring_pos[a:b], model.freqs,
                                pool.swa[layer])
        ratio = cfg.compress_ratios[layer]
        if ratio == abi.C4_RATIO:
            for a in range(0, phys4.numel(), chunk_rows):
                b = min(phys4.numel(), a + chunk_rows)
                model._store_c4(layer, rand_rows(b - a), phys4[a:b], pos4[a:b])
            for a in range(0, phys4.numel(), chunk_rows):
                b = min(phys4.numel(), a + chunk_rows)
                krows = torch.empty(b - a, cfg.index_dim, device=dev).normal_(generator=gen)
                idx_ops.index_key_store(krows, phys4[a:b], pool.index_keys[layer], pool.index_scales[layer])
        elif ratio == abi.C128_RATIO:
            for a in range(0, phys2.numel(), chunk_rows):
                b = min(phys2.numel(), a + chunk_rows)
                kv_ops.native_store(rand_rows(b - a), lw["c_norm"], eps, phys2[a:b], pos2[a:b], model.freqs,
                                    pool.c128_native[layer])
    engine.running.extend(reqs)
    return reqs

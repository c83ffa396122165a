"""CPU oracle experiment: Packed vs Native C4 records on one MLA layer (fp32 torch, seed-driven).

    python -m packmla.bench.oracle_experiment [--batch 4 --heads 64 --context 8192 --topk 512 --seed 0]

Setup (the reference's CPU format experiment): latent rows ~ N(0, 1) of width 512 (448 NoPE coordinates stored
as E4M3 with per-64-coordinate UE8M0 scales, 64 RoPE coordinates in BF16); queries ~ N(0, 1) / sqrt(576);
a context of `context` tokens compressed 4:1 into C4 records; a fixed seeded mask keeps all 64 RoPE
coordinates plus 192 seeded NoPE coordinates (256 of 512).  Every record is written as a Native 584 B
record and as a Packed 328 B record (same mask for every record; the data-dependent TopMag mask is
reported beside it for contrast), each query attends over its top-k
records by score (the sum over heads of the query-record logits on the Native rows), and the outputs are
compared: Packed vs Native, and both vs the unquantized fp32 rows.  Byte and capacity accounting come
from the ABI and `plan_capacity`.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from ..config import EngineConfig, ModelConfig
from ..formats import abi, codec
from ..kv.pool import plan_capacity
from ..oracle import attention as oracle


def seeded_mask(seed: int) -> torch.Tensor:
    """All 64 RoPE coordinates + 192 NoPE coordinates chosen by a seeded permutation."""
    g = torch.Generator().manual_seed(seed)
    mask = torch.zeros(abi.LATENT_DIM, dtype=torch.bool)
    mask[abi.NOPE_DIM:] = True
    mask[torch.randperm(abi.NOPE_DIM, generator=g)[:192]] = True
    return mask


def run(batch: int = 4, heads: int = 64, context: int = 8192, topk: int = 512, seed: int = 0) -> dict:
    g = torch.Generator().manual_seed(seed)
    records = context // abi.C4_RATIO
    raw = torch.randn(records, abi.LATENT_DIM, generator=g)
    weight = torch.ones(abi.LATENT_DIM)
    eps = 1e-6
    table = codec.rope_table(context)
    pos = torch.arange(records) * abi.C4_RATIO
    freqs = table[pos]
    mask = seeded_mask(seed)
    native_rec = codec.native_encode(raw, weight, eps, freqs)
    native_rows = codec.native_decode(native_rec)
    vals, bits, scs = codec.packed_encode(raw, weight, eps, mask=mask.expand(records, -1).contiguous())
    packed_rows = codec.packed_read(vals, bits, scs, freqs)
    tv, tb, ts = codec.packed_encode(raw, weight, eps)  # TopMag: the 256 largest |x| of every record
    topmag_rows = codec.packed_read(tv, tb, ts, freqs)
    exact_rows = codec.rotate_tail(codec.rms_normalize(raw, weight, eps), freqs)  # bf16 norm, no quantization
    q = torch.randn(batch, heads, abi.LATENT_DIM, generator=g) / math.sqrt(576.0)
    sink = torch.full((heads,), -math.inf)  # no sink in this experiment
    scale = oracle.default_scale()
    errs = {"packed_vs_native": [], "native_vs_exact": [], "packed_vs_exact": [], "topmag_vs_native": []}
    for b in range(batch):
        score = (q[b] @ native_rows.T).sum(0)
        sel = score.topk(topk).indices
        outs = {}
        for name, rows in (("native", native_rows), ("packed", packed_rows), ("exact", exact_rows),
                           ("topmag", topmag_rows)):
            outs[name] = oracle.attend(q[b], rows[sel], sink, scale)[0]
        for key, (a, ref) in (("packed_vs_native", ("packed", "native")), ("native_vs_exact", ("native", "exact")),
                              ("packed_vs_exact", ("packed", "exact")), ("topmag_vs_native", ("topmag", "native"))):
            errs[key].append(float((outs[a] - outs[ref]).norm() / outs[ref].norm()))
    cfg = ModelConfig()
    budget = 30 << 30
    native_cap = plan_capacity(cfg, EngineConfig(kv_cache_format="native"), budget).max_total_tokens
    direct_cap = plan_capacity(cfg, EngineConfig(kv_cache_format="direct"), budget).max_total_tokens
    return {
        "batch": batch, "heads": heads, "context": context, "records": records, "topk": topk, "seed": seed,
        "mask": {"rope_kept": int(mask[abi.NOPE_DIM:].sum()), "nope_kept": int(mask[:abi.NOPE_DIM].sum())},
        "relative_output_error": {k: {"mean": sum(v) / len(v), "max": max(v)} for k, v in errs.items()},
        "bytes": {"native_record": abi.NATIVE_RECORD_BYTES, "packed_record": abi.PACKED_RECORD_BYTES,
                  "native_layer": records * abi.NATIVE_RECORD_BYTES, "packed_layer": records * abi.PACKED_RECORD_BYTES,
                  "packed_over_native": abi.PACKED_RECORD_BYTES / abi.NATIVE_RECORD_BYTES},
        "capacity_tokens_30GiB": {"native": native_cap, "direct": direct_cap, "ratio": direct_cap / native_cap},
    }


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--heads", type=int, default=64)
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--topk", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    print(json.dumps(run(a.batch, a.heads, a.context, a.topk, a.seed), indent=2))


if __name__ == "__main__":
    main()

"""Per-kernel breakdown of the serving decode step (one GPU).

    python -m packmla.bench.step_breakdown [--concurrency 8] [--prompt-len 32768] [--steps 8]

Builds the engine of `bench.py` (V4-Flash shape, random init, Direct KV), prefills `--concurrency`
synthetic prompts through `Engine.step()` so every request decodes at its full context, then runs
`--steps` decode steps eagerly (graphs off, so each kernel is seen on its own) under the PyTorch
profiler and sums the device time of every kernel.  Prints one JSON object: the eager step's summed
kernel time, the graph-replay step time of the same batch (CUDA events), and the kernels grouped into
families with their time per step and share.  Shares are what this reports; the profiler's absolute
times are close to, not equal to, unprofiled kernel times.
"""
from __future__ import annotations

import argparse
import json
import re
import time

# kernel-name patterns -> family (first match wins)
FAMILIES = [
    ("attention (sparse MLA decode)", r"sparse_mla_decode|mla_combine"),
    ("MoE experts (MXFP4)", r"mx_expert|moe_fp4|mx_quant|moe_route|moe_gather|moe_place|moe_count|moe_plan"),
    ("indexer", r"index_logits|index_topk|index_key"),
    ("dense projections, MXFP8 (packmla)", r"dense_mx|dense_quant"),
    ("routing", r"route_topk"),
    ("dense GEMM (cuBLAS)", r"nvjet|gemm|cutlass|sm90|sm100|cublas|Kernel2"),
    ("norms / RoPE / SiLU (packmla)", r"add_rmsnorm|rope_q|silu_mul|rmsnorm"),
    ("KV stores / compressor (packmla)", r"native_store|packed_store|comp_pool"),
    ("sampling / torch elementwise", r"elementwise|reduce|argmax|gather|scatter|index|copy|fill|Memcpy|Memset"),
]


def family(name: str) -> str:
    for fam, pat in FAMILIES:
        if re.search(pat, name):
            return fam
    return "other"


def _families(prof, per: int, top: int) -> tuple[float, dict, list]:
    per_kernel: dict[str, float] = {}
    for ev in prof.key_averages():
        t = getattr(ev, "self_device_time_total", None)
        if t is None:
            t = ev.self_cuda_time_total
        if t > 0:
            per_kernel[ev.key] = per_kernel.get(ev.key, 0.0) + t / per
    total = sum(per_kernel.values())
    fams: dict[str, float] = {}
    for k, v in per_kernel.items():
        fams[family(k)] = fams.get(family(k), 0.0) + v
    return total, ({k: {"us": round(v, 1), "share": round(v / total, 4)}
                    for k, v in sorted(fams.items(), key=lambda kv: -kv[1])}), (
        [{"name": k[:90], "us": round(v, 1), "share": round(v / total, 4)}
         for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1])[:top]])


def prefill_breakdown(args, cfg, device) -> dict:
    """Kernel time of one 8192-token prefill chunk (the third of one request, eager, under the profiler)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from ..engine.engine import SamplingParams
    from ..ops import check_errors
    from ..parallel.comm import TPComm
    from .engine_setup import build_engine

    eng, _ = build_engine(cfg, device, 0, 1, TPComm(), 1, args.prompt_len, args.output_len, args.kv_format,
                          prefix_cache=False)
    gen = torch.Generator().manual_seed(0)
    eng.add_request(torch.randint(0, cfg.vocab_size, (args.prompt_len,), generator=gen).tolist(),
                    SamplingParams(max_new_tokens=1))
    for _ in range(2):
        eng.step()
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        s.record()
        eng.step()
        e.record()
        torch.cuda.synchronize(device)
    check_errors(device)
    total, fams, kernels = _families(prof, 1, args.top)
    out = {"case": "prefill_chunk_breakdown", "chunk_tokens": 8192, "positions": [16384, 24576],
           "kv_format": args.kv_format, "chunk_ms_profiled": round(s.elapsed_time(e), 2),
           "kernel_ms": round(total / 1e3, 2), "families": fams, "kernels": kernels}
    print(json.dumps(out), flush=True)
    return out


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--concurrency", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=32768)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--kv-format", default="direct", choices=["direct", "native"])
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--dense-format", default="bf16", choices=["bf16", "fp8"])
    ap.add_argument("--top", type=int, default=25, help="kernels listed individually")
    ap.add_argument("--phase", default="decode", choices=["decode", "prefill"],
                    help="prefill: one request alone, its third 8192-token chunk profiled (positions 16k-24k)")
    args = ap.parse_args(argv)

    import torch
    from torch.profiler import ProfilerActivity, profile

    from ..config import ModelConfig
    from ..engine.engine import SamplingParams
    from ..ops import check_errors
    from ..parallel.comm import TPComm
    from .engine_setup import build_engine

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = ModelConfig(dense_format=args.dense_format)
    C = args.concurrency
    if args.phase == "prefill":
        return prefill_breakdown(args, cfg, device)
    eng, _ = build_engine(cfg, device, 0, 1, TPComm(), C, args.prompt_len, args.output_len, args.kv_format)
    eng.runner.capture()
    gen = torch.Generator().manual_seed(0)
    params = SamplingParams(max_new_tokens=args.output_len, temperature=0.0, ignore_eos=True)
    for _ in range(C):
        eng.add_request(torch.randint(0, cfg.vocab_size, (args.prompt_len,), generator=gen).tolist(), params)
    t0 = time.time()
    # prefill every prompt (chunks alternate with decode steps of the requests already running)
    def prefilling() -> bool:
        return bool(eng.waiting) or any(r.prefilled < len(r.prompt) for r in eng.running)

    while eng.has_work() and prefilling():
        eng.step()
    torch.cuda.synchronize(device)
    prefill_s = time.time() - t0
    for _ in range(3):  # warm decode steps (graph replays)
        eng.step()
    # graph-replay step time of this batch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        eng.step()
    e.record()
    torch.cuda.synchronize(device)
    graph_ms = s.elapsed_time(e) / args.steps
    # the same steps eagerly under the profiler
    eng.runner.enabled = False
    eng.step()
    torch.cuda.synchronize(device)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            eng.step()
        torch.cuda.synchronize(device)
    eng.runner.enabled = True
    check_errors(device)
    per_kernel: dict[str, float] = {}
    for ev in prof.key_averages():
        t = getattr(ev, "self_device_time_total", None)
        if t is None:
            t = ev.self_cuda_time_total
        if t > 0:
            per_kernel[ev.key] = per_kernel.get(ev.key, 0.0) + t / args.steps  # us per step
    total = sum(per_kernel.values())
    fams: dict[str, float] = {}
    for k, v in per_kernel.items():
        fams[family(k)] = fams.get(family(k), 0.0) + v
    out = {
        "case": "decode_step_breakdown", "concurrency": C, "prompt_len": args.prompt_len,
        "kv_format": args.kv_format, "dense_format": args.dense_format, "steps": args.steps, "prefill_s": round(prefill_s, 1),
        "graph_step_ms": round(graph_ms, 3), "eager_kernel_ms_per_step": round(total / 1e3, 3),
        "families": {k: {"us_per_step": round(v, 1), "share": round(v / total, 4)}
                     for k, v in sorted(fams.items(), key=lambda kv: -kv[1])},
        "kernels": [{"name": k[:90], "us_per_step": round(v, 1), "share": round(v / total, 4)}
                    for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1])[:args.top]],
    }
    print(json.dumps(out), flush=True)
    eng.runner.release()
    return out


if __name__ == "__main__":
    main()

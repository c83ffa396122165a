"""Serving benchmark of the flagship path (driver contract), BASELINE config 3.

    python bench.py [--gpus N --steps K --warmup W]                  (N=1)
    torchrun --nproc-per-node N bench.py --gpus N --steps K --warmup W

Workload: the random-init DeepSeek-V4-Flash-shape model (43 layers, 64 heads x 512 latent, C4/C128 compressed
sparse attention, 256 MXFP4 routed experts + 1 shared) served in Direct mode (Packed 328 B KV) with TP = EP = N.
Synthetic uniform-random-token prompts of 32768 tokens, 256 output tokens each (greedy, EOS ignored), at a
concurrency of C requests: C warm-up requests, the prefix cache flushed, then 3C measured requests, all through
`Engine.step()` (chunked prefill of 8192 tokens, prefill chunks alternating with decode steps, CUDA-graph
decode), as the reference's serving client runs them (scripts/local/bench-serving.sh:153-192).  C defaults to
8 / 8 / 24 / 40 requests at 1 / 2 / 4 / 8 GPUs (the config's concurrency levels).

* value: decode output tokens/s of the measured phase on the device clock: output tokens produced by decode
  steps / the summed CUDA-event time of those steps (graph replay of all 43 layers + sampling); max over ranks.
* e2e:   output tokens/s of the measured phase end to end: every output token (the first comes from its
  prefill) / wall time of the phase, which includes the host -> device copy of every prompt chunk from pinned
  memory, all prefill chunks, all decode steps and the device -> host read of every sampled token; max over
  ranks.
* steps / ms_per_step: the measured phase's decode steps and their mean device time.  The protocol fixes the
  amount of work (3C requests of 32768 + 256 tokens), so --steps and --warmup do not change it; they are
  recorded as `steps_requested` / `warmup` (W must be >= 3; the warm-up phase runs C full requests).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode output tok/s (32k in/256 out)"


def build_identity() -> dict:
    """The source identity of this run (packmla.utils.provenance): commit, modified paths, the compiled
    sources' digest, the library's sha256 and whether it was built from those sources."""
    from packmla.utils.provenance import source_identity

    ident = source_identity()
    return {"git_sha": ident["git_commit"], "modified": ident["modified"], "csrc_sha256": ident["csrc_sha256"],
            "extension_sha256": (ident["library"]["sha256"] or "")[:16] or None,
            "library_matches_sources": ident["library_matches_sources"]}


def reference_arm(args) -> None:
    out = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus,
           "unavailable": ("the reference (winstonxcai/flash-optimizations) is not installable: no setup.py or "
                           "pyproject.toml, and its SGLang/FlashMLA runtime lives in git submodules that are empty "
                           "in the mounted checkout, so no public API exists to run")}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(out), flush=True)


def run_phase(eng, prompts: list[list[int]], params, comm, device, timed: bool) -> dict:
    """Submit all prompts (the engine keeps at most C running) and step until they finish."""
    import torch

    cuda = device.type == "cuda"
    eng.step_events = [] if timed else None
    rids = [eng.add_request(p, params) for p in prompts]
    comm.barrier()
    if cuda:
        torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    h2d = d2h = 0
    n_steps = 0
    while eng.has_work():
        eng.step()
        n_steps += 1
        h2d += eng.h2d_bytes_last
        d2h += eng.d2h_bytes_last
        eng.h2d_bytes_last = eng.d2h_bytes_last = 0
    if cuda:
        torch.cuda.synchronize(device)
    wall = time.perf_counter() - t0
    comm.barrier()
    out_tokens = sum(len(eng.result(r).output_ids) for r in rids if eng.owns(r))  # this rank's requests
    stats = {"wall_s": wall, "engine_steps": n_steps, "out_tokens": out_tokens, "h2d": h2d, "d2h": d2h}
    if timed:
        dec_ms = pre_ms = 0.0
        n_dec = 0
        for kind, s, e in eng.step_events:
            ms = s.elapsed_time(e)
            if kind == "decode":
                dec_ms += ms
                n_dec += 1
            else:
                pre_ms += ms
        stats.update(decode_ms=dec_ms, prefill_ms=pre_ms, decode_steps=n_dec)
        eng.step_events = None
    return stats


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20, help="recorded only: the protocol fixes the work")
    ap.add_argument("--warmup", type=int, default=5, help="recorded only (>= 3): the warm-up phase is C requests")
    ap.add_argument("--impl", default="packmla", choices=["packmla", "reference"])
    ap.add_argument("--concurrency", type=int, default=None,
                    help="concurrent requests C (default 8 / 8 / 24 / 40 at 1 / 2 / 4 / 8 GPUs)")
    ap.add_argument("--prompt-len", type=int, default=32768)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--kv-format", default="direct", choices=["direct", "native", "fp4-native", "fp4-direct"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dense-format", default="bf16", choices=["bf16", "fp8"],
                    help="dense projections: BF16 (cuBLAS) or MXFP8 weights (packmla's tcgen05 GEMM)")
    ap.add_argument("--collectives", default="auto", choices=["auto", "fused", "nccl"],
                    help="TP all-reduces: packmla's fused GEMM+all-reduce kernels over NVLink, or NCCL; auto = fused "
                         "at the world sizes the fused kernels were validated on (2 and 4), NCCL otherwise")
    ap.add_argument("--dp-attention", default="auto", choices=["auto", "on", "off"],
                    help="DP attention (each rank serves C/N requests with every head, MoE tokens exchanged by "
                         "all-gather / reduce-scatter) or TP attention; auto = TP")
    ap.add_argument("--oproj-gemm", default="auto", choices=["auto", "fused", "library"],
                    help="with fused collectives: projection inside the all-reduce kernel, cuBLAS first, or "
                         "by token count")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch

    from packmla.bench.engine_setup import DEFAULT_CONCURRENCY, build_engine
    from packmla.bench.timing import ClockSampler
    from packmla.config import EngineConfig, ModelConfig
    from packmla.engine.engine import SamplingParams
    from packmla.kv.pool import plan_capacity
    from packmla.ops import _ext, check_errors
    from packmla.parallel.comm import TPComm, init_from_env

    rank, world, local = init_from_env("nccl")
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = ModelConfig(dense_format=args.dense_format)
    C = args.concurrency or DEFAULT_CONCURRENCY.get(world, 8 * world)
    dp = world > 1 and args.dp_attention == "on"
    if dp and C % world:
        raise SystemExit(f"--dp-attention: concurrency {C} must be a multiple of {world}")
    if args.collectives == "auto":
        args.collectives = "fused" if world in (2, 4) and not dp else "nccl"
    if dp and args.collectives == "fused":
        raise SystemExit("--dp-attention exchanges MoE tokens over NCCL: use --collectives nccl")
    if world > 1 and args.collectives == "fused":
        from packmla.parallel.fused import FusedComm

        comm = FusedComm(device, cfg.hidden_size, gemm=args.oproj_gemm)
    else:
        comm = TPComm()
    t0 = time.time()
    eng, max_context = build_engine(cfg, device, rank, world, comm, C, args.prompt_len, args.output_len,
                                    args.kv_format, args.seed, dp_attention=dp)
    eng.runner.capture()
    torch.cuda.synchronize(device)
    # kernel launches of one decode step (an eager forward at the dummy slot, counted by the extension proxy)
    ext = _ext.ext()
    ext.launches, ext.enabled = 0, True
    eng.runner._forward(eng.runner.max_b)
    ext.enabled = False
    launches_per_decode = ext.launches
    eng.pool.comp_state_reset(eng.dummy_slot)
    torch.cuda.synchronize(device)
    check_errors(device)
    t_build = time.time() - t0

    gen = torch.Generator().manual_seed(args.seed)  # same prompts on every rank (TP lockstep)

    def prompts(n):
        return [torch.randint(0, cfg.vocab_size, (args.prompt_len,), generator=gen).tolist() for _ in range(n)]

    params = SamplingParams(max_new_tokens=args.output_len, temperature=0.0, ignore_eos=True)
    # ---------------- warm-up phase: C requests, then the prefix cache is flushed
    run_phase(eng, prompts(C), params, comm, device, timed=False)
    eng.flush_cache()
    check_errors(device)
    # ---------------- measured phase: 3C requests at concurrency C
    measured = prompts(3 * C)
    ext.launches, ext.enabled = 0, True  # prefill chunks run eagerly: their launches are counted as they go
    with ClockSampler(local) as clk:
        st = run_phase(eng, measured, params, comm, device, timed=True)
    ext.enabled = False
    prefill_launches = ext.launches
    check_errors(device)

    dec_ms = comm.max_over_ranks(st["decode_ms"], device)
    wall_s = comm.max_over_ranks(st["wall_s"], device)
    pre_ms = comm.max_over_ranks(st["prefill_ms"], device)
    n_req = 3 * C
    out_tokens = int(comm.sum_over_ranks(st["out_tokens"], device)) if dp else st["out_tokens"]
    dec_tokens = out_tokens - n_req  # each request's first token comes from its prefill
    value = dec_tokens / (dec_ms / 1000.0)
    e2e = out_tokens / wall_s
    n_dec = max(1, st["decode_steps"])
    native_cap = plan_capacity(cfg, EngineConfig(kv_cache_format="native"), 1 << 40).max_total_tokens
    direct_cap = plan_capacity(cfg, EngineConfig(kv_cache_format="direct"), 1 << 40).max_total_tokens
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": st["decode_steps"],
        "steps_requested": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dec_ms / n_dec, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": ("synthetic: uniform-random-token prompts, random-init weights of the model's architecture "
                 "(no checkpoint or dataset offline)"),
        "impl": "packmla",
        "config": {
            "model": "DeepSeek-V4-Flash-shape (43 layers, hidden 4096, 64 heads x 512 latent, C4/C128 CSA, "
                     "256 MXFP4 routed experts top-8 + 1 shared), random init",
            "global_batch": C,
            "concurrency": C,
            "seq_len": args.prompt_len,
            "output_len": args.output_len,
            "requests_warmup": C,
            "requests_measured": n_req,
            "prefix_cache": "on, flushed between the warm-up and measured phases",
            "chunked_prefill": 8192,
            "parallelism": (f"dp{world}-attention ep{world}" if dp else f"tp{world}ep{world}"),
            "collectives": (f"{args.collectives}/oproj-{args.oproj_gemm}" if args.collectives == "fused"
                            else args.collectives) if world > 1 else "none",
            "kv_cache_format": args.kv_format,
            "dense_format": args.dense_format,
            "l2": ("inputs larger than L2: every decode step streams the routed experts its tokens select (up to "
                   "~108 GB / N of MXFP4 weights) and each request's selected KV rows of 43 layers"),
            "vs_baseline_note": ("the reference publishes no 32k/256 decode number (its README's 32k/256/C2 "
                                 "smoke has no recorded result); nearest published: 128k/8k C24 589.9 output "
                                 "tok/s on 4xH100 TP4"),
            "kv_capacity_vs_native_planned": round(direct_cap / native_cap, 4),
        },
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": int(st["h2d"] / max(1, st["engine_steps"])),
                "d2h_bytes_per_step": int(st["d2h"] / max(1, st["engine_steps"])),
                "wall_s": round(wall_s, 2), "engine_steps": st["engine_steps"],
                "prefill_tokens_per_s_device": round(n_req * args.prompt_len / (pre_ms / 1000.0), 1),
                "prefill_device_s": round(pre_ms / 1000.0, 2), "decode_device_s": round(dec_ms / 1000.0, 2)},
        "gpu_launches": prefill_launches + launches_per_decode * st["decode_steps"],
        "clocks": clk.summary(),
        "setup_s": round(t_build, 1),
        "build": build_identity(),
    }
    # graphs hold NCCL calls under TP: drop every reference and destroy them before the group
    eng.runner.release()
    import gc

    gc.collect()
    torch.cuda.synchronize(device)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import threading

        import torch.distributed as dist

        dist.barrier()
        if hasattr(comm, "close"):
            comm.close()
        # bounded teardown: a communicator that does not shut down must not hold the GPUs
        t = threading.Thread(target=dist.destroy_process_group, daemon=True)
        t.start()
        t.join(60)
        sys.stdout.flush()
        os._exit(0 if not t.is_alive() else 3)


if __name__ == "__main__":
    main()

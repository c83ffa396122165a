"""Decode-throughput benchmark of the flagship serving path (driver contract).

    python bench.py [--gpus N --steps K --warmup W]                  (N=1)
    torchrun --nproc-per-node N bench.py --gpus N --steps K --warmup W

Metric: decode output tokens/s at 32k input / 256 output for the random-init
DeepSeek-V4-Flash-shape model (43 layers, 64 heads x 512 latent, C4/C128 compressed sparse
attention, 256 MXFP4 routed experts + 1 shared), Direct (Packed 328 B) KV, TP=N attention and
EP=N experts.  Every request holds a 32768-token context written by the engine's own store
kernels (synthetic random latents, no prefill), then decodes one token per step.

* value: device time of K decode steps (CUDA-graph replay of all 43 layers + sampling, tokens fed
  back on device), CUDA events, barrier + synchronize on both sides, max over ranks.
* e2e:   K steps through the public API `Engine.step()`: pinned host -> device copy of the step's
  inputs, graph replay, device -> host read of the sampled tokens, host bookkeeping; wall clock,
  max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode output tok/s (32k in/256 out)"


def build_identity() -> dict:
    """git commit (when the checkout has one) and sha256 of the loaded extension."""
    import glob
    import hashlib
    import subprocess

    out = {}
    try:
        out["git_sha"] = subprocess.run(["git", "rev-parse", "HEAD"], cwd=ROOT, capture_output=True, text=True,
                                        timeout=10).stdout.strip() or None
    except (OSError, subprocess.SubprocessError):
        out["git_sha"] = None
    so = sorted(glob.glob(os.path.join(ROOT, "packmla", "_C*.so")))
    if so:
        with open(so[0], "rb") as f:
            out["extension_sha256"] = hashlib.sha256(f.read()).hexdigest()[:16]
    return out


def reference_arm(args) -> None:
    out = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus,
           "unavailable": ("the reference (winstonxcai/flash-optimizations) is not installable: no setup.py or "
                           "pyproject.toml, and its SGLang/FlashMLA runtime lives in git submodules that are empty "
                           "in the mounted checkout, so no public API exists to run")}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(out), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48)
    ap.add_argument("--warmup", type=int, default=6)
    ap.add_argument("--impl", default="packmla", choices=["packmla", "reference"])
    ap.add_argument("--concurrency", type=int, default=40, help="concurrent requests per GPU (weak scaling)")
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--kv-format", default="direct", choices=["direct", "native"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--collectives", default="auto", choices=["auto", "fused", "nccl"],
                    help="TP all-reduces: packmla's fused GEMM+all-reduce kernels over NVLink, or NCCL; auto = fused "
                         "at the world sizes the fused kernels were validated on (2), NCCL otherwise")
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

    from packmla.bench.synthetic import fill_synthetic
    from packmla.bench.timing import ClockSampler, time_device
    from packmla.config import EngineConfig, ModelConfig
    from packmla.engine.engine import Engine
    from packmla.kv.pool import bytes_per_full_token, fixed_bytes, plan_capacity
    from packmla.ops import _ext, check_errors
    from packmla.parallel.comm import TPComm, init_from_env

    rank, world, local = init_from_env("nccl")
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = ModelConfig()
    C = args.concurrency * world
    if args.collectives == "auto":
        args.collectives = "fused" if world == 2 else "nccl"
    if world > 1 and args.collectives == "fused":
        from packmla.parallel.fused import FusedComm

        comm = FusedComm(device, cfg.hidden_size, gemm=args.oproj_gemm)
    else:
        comm = TPComm()
    steps_total = args.warmup + 2 * args.steps + 4
    if steps_total > args.output_len:
        raise SystemExit(f"warmup + 2*steps + 4 = {steps_total} exceeds the {args.output_len}-token output")
    max_context = args.context + args.output_len + 256
    ecfg = EngineConfig(kv_cache_format=args.kv_format, tp=world, ep=world, max_running_requests=C,
                        cuda_graph_bs=[C], chunked_prefill_size=8192)
    pages_per_req = math.ceil(max_context / 256)
    bpt = bytes_per_full_token(cfg, args.kv_format, ecfg.swa_full_tokens_ratio)
    kv_bytes = int((C * pages_per_req + 8) * 256 * bpt) + fixed_bytes(cfg, C + 1) + (64 << 20)

    t0 = time.time()
    eng = Engine.build(cfg, ecfg, device, rank, world, comm, max_context=max_context, max_requests=C,
                       kv_bytes=kv_bytes, seed=args.seed)
    torch.cuda.synchronize(device)
    t_build = time.time() - t0
    fill_synthetic(eng, C, args.context, args.output_len, seed=args.seed + rank * 0)
    torch.cuda.synchronize(device)
    check_errors(device)
    # capture the decode graph; count our kernel launches per step while recording it
    ext = _ext.ext()
    ext.enabled, ext.launches = False, 0
    eng.runner.capture([C])  # includes an eager warm-up forward
    torch.cuda.synchronize(device)
    # recapture once with counting on (same graph shape; replaces the first)
    ext.enabled = True
    eng.runner.graphs.clear()
    eng.runner.capture([C])
    ext.enabled = False
    launches_per_step = ext.launches // 2  # warm-up forward + captured forward
    check_errors(device)

    for _ in range(args.warmup):  # warm-up through the public API
        eng.step()
    torch.cuda.synchronize(device)
    check_errors(device)

    # ---------------- device-timed decode (graph replays, tokens fed back on device)
    runner = eng.runner
    b = len(eng.running)
    for i, r in enumerate(eng.running):
        runner.tokens[i] = r.output_ids[-1]
        runner.positions[i] = r.context_len - 1
        runner.slots[i] = r.slot
    g = runner.graphs[runner.bucket(b)]

    def device_step():
        g.replay()
        runner.tokens[:b].copy_(runner.out_tokens[:b])
        runner.positions[:b].add_(1)

    comm.barrier()
    with ClockSampler(local) as clk:
        dev_ms = time_device(device_step, args.steps, device)
    comm.barrier()
    dev_ms = comm.max_over_ranks(dev_ms, device)
    last = runner.out_tokens[:b].tolist()
    for r, tok in zip(eng.running, last):
        r.output_ids.extend([tok] * args.steps)
    check_errors(device)

    # ---------------- end-to-end through Engine.step()
    comm.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clk_e2e:  # its own clock record: the two windows can run at different clocks
        t1 = time.perf_counter()
        for _ in range(args.steps):
            eng.step()
        torch.cuda.synchronize(device)
        e2e_s = time.perf_counter() - t1
    comm.barrier()
    e2e_s = comm.max_over_ranks(e2e_s, device)
    check_errors(device)

    native_cap = plan_capacity(cfg, EngineConfig(kv_cache_format="native"), 1 << 40).max_total_tokens
    direct_cap = plan_capacity(cfg, EngineConfig(kv_cache_format="direct"), 1 << 40).max_total_tokens
    value = C * args.steps / (dev_ms / 1000.0)
    e2e = C * args.steps / e2e_s
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-token requests; 32k-token contexts written as random latents by the store kernels)",
        "impl": "packmla",
        "config": {
            "model": "DeepSeek-V4-Flash-shape (43 layers, hidden 4096, 64 heads x 512 latent, C4/C128 CSA, "
                     "256 MXFP4 routed experts top-8 + 1 shared), random init",
            "global_batch": C,
            "concurrency_per_gpu": args.concurrency,
            "seq_len": args.context,
            "output_len": args.output_len,
            "parallelism": f"tp{world}ep{world}",
            "collectives": (f"{args.collectives}/oproj-{args.oproj_gemm}" if args.collectives == "fused"
                            else args.collectives) if world > 1 else "none",
            "kv_cache_format": args.kv_format,
            "l2": "inputs larger than L2 (all ~150 GB of weights and the KV cache are read every step)",
            "kv_capacity_vs_native": round(direct_cap / native_cap, 4),
        },
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": eng.h2d_bytes_last,
                "d2h_bytes_per_step": eng.d2h_bytes_last, "ms_per_step": round(e2e_s * 1000 / args.steps, 4),
                "clocks": clk_e2e.summary()},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
        "setup_s": round(t_build, 1),
        "build": build_identity(),
    }
    # graphs hold NCCL calls under TP: drop every reference and destroy them before the group
    del g, device_step
    eng.runner.release()
    import gc

    gc.collect()
    torch.cuda.synchronize(device)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import os
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

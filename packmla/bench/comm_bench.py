"""Per-call device time of the TP collectives: packmla's fused kernels vs cuBLAS + NCCL.

    torchrun --nproc-per-node N -m packmla.bench.comm_bench [--tokens B ...]
    python -m packmla.bench.comm_bench [--tokens B ...]          (one GPU: the kernels at world 1)

Cases per token count B (decode batch of all ranks' requests):
  o_proj   Y = sum_r X_r W_r^T, X_r [B, 8192/N], W_r [4096, 8192/N] bf16 (attention output projection)
           fused: gemm_allreduce (one kernel);  baseline: torch.mm + dist.all_reduce (NCCL)
  moe_sum  Y = sum_r (F_r + A_r), F fp32 / A bf16 [B, 4096] (routed + shared expert outputs)
           fused: allreduce (one kernel);       baseline: add + cast + dist.all_reduce
Each case replays a CUDA graph of R calls; time = CUDA events / calls, max over ranks.  Roofline of
a call: max(weight bytes / measured HBM copy bandwidth, NVLink bytes per rank / 770 GB/s).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _graph_time(fn, calls: int, replays: int, warm: int = 3) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (calls * replays)
    g.reset()
    t = torch.tensor([us], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="*", default=None)
    ap.add_argument("--calls", type=int, default=20)
    ap.add_argument("--replays", type=int, default=20)
    ap.add_argument("--splits", type=int, nargs="*", default=[0])
    ap.add_argument("--modes", nargs="*", default=["auto"], choices=["auto", "one", "two"])
    args = ap.parse_args()
    from ..parallel.comm import init_from_env
    from ..parallel.fused import FusedComm, choose_splits, use_one_shot
    from ..ops._ext import check_errors

    rank, world, local = init_from_env("nccl")
    if not dist.is_initialized():  # one process without torchrun: a one-rank group (the kernels run at world 1)
        import socket

        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{port}",
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    hidden, o_in = 4096, 8192
    K = o_in // world
    comm = FusedComm(dev, hidden)
    try:
        hbm = json.load(open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")))["hbm_gbs"]
    except (OSError, KeyError, ValueError):
        hbm = 6650.0
    tokens = args.tokens or [1, 40 * world, 320]
    g = torch.Generator(device=dev).manual_seed(rank)
    rows = []
    for B in tokens:
        x = torch.randn(B, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(hidden, K, device=dev, generator=g) / K ** 0.5).bfloat16()
        f = torch.randn(B, hidden, device=dev, generator=g)
        a = torch.randn(B, hidden, device=dev, generator=g).bfloat16()

        def base_oproj():
            y = x @ w.T
            dist.all_reduce(y)

        def base_moe():
            y = (f + a.float()).bfloat16()
            dist.all_reduce(y)

        t_base = _graph_time(base_oproj, args.calls, args.replays)
        t_cublas_ar = _graph_time(lambda: comm.all_reduce_sum(None, x @ w.T), args.calls, args.replays)
        t_base_moe = _graph_time(base_moe, args.calls, args.replays)
        out_bytes = B * hidden * 2
        for mode in args.modes:
            one = None if mode == "auto" else (mode == "one")
            shot = use_one_shot(world, out_bytes) if one is None else one
            link = ((world - 1) * out_bytes if shot else 2 * (world - 1) / world * out_bytes) / (NVLINK_GBS * 1e3)
            for sp in args.splits:
                s = sp or choose_splits(hidden, K, B)
                if K % (64 * s) or (hidden // 256) * -(-B // 128) * s > comm.num_sms or world + s > comm.max_src:
                    continue
                t_f = _graph_time(lambda: comm.gemm_all_reduce(x, w, s, one), args.calls, args.replays)
                prof = torch.zeros(8, dtype=torch.int64, device=dev)
                comm.gemm_all_reduce(x, w, s, one, prof)
                torch.cuda.synchronize()
                pv = prof.tolist()
                n = max(pv[3], 1)
                roof = max(hidden * K * 2 / (hbm * 1e3), link)
                rows.append({"case": "o_proj", "tokens": B, "K": K, "splits": s, "one_shot": shot,
                             "fused_us": round(t_f, 2), "cublas_nccl_us": round(t_base, 2),
                             "cublas_fused_ar_us": round(t_cublas_ar, 2),
                             "speedup": round(t_base / t_f, 3), "roofline_us": round(roof, 2),
                             "fraction_of_roofline": round(roof / t_f, 3),
                             "phases_us_mean": {"gemm": round(pv[0] / n / 1e3, 2), "push": round(pv[1] / n / 1e3, 2),
                                                "reduce": round(pv[2] / n / 1e3, 2)},
                             "cta_max_us": round(pv[4] / 1e3, 2)})
            t_moe = _graph_time(lambda: comm.all_reduce_sum(f, a, one), args.calls, args.replays)
            rows.append({"case": "moe_sum", "tokens": B, "one_shot": shot, "fused_us": round(t_moe, 2),
                         "nccl_us": round(t_base_moe, 2), "speedup": round(t_base_moe / t_moe, 3),
                         "roofline_us": round(link, 2)})
    check_errors(dev)
    if rank == 0:
        for r in rows:
            print(json.dumps({"world": world, **r}), flush=True)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

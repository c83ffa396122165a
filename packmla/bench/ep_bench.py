"""Expert-parallel MoE layer of the V4-Flash shape: dispatch / local experts / combine, per-phase time.

    torchrun --nproc-per-node N -m packmla.bench.ep_bench [--tokens 4096 --iters 5]
    python -m packmla.bench.ep_bench                # one GPU: all experts local, no exchange

Workload: every rank holds `tokens` tokens (hidden 4096, BF16) routed top-8 over 256 routed experts from
seeded Gaussian gate logits (weights: softmax over the chosen 8), plus one shared expert (intermediate
2048) on the rank's own tokens.  Each rank owns 256 / N MXFP4 experts; routed pairs go to the owner
through `torch.distributed.all_to_all_single` (NCCL), the owner runs packmla's MXFP4 x MXFP8 tcgen05
expert kernel on what it received, and BF16 outputs come back for the weighted sum.  Phases are timed
with CUDA events around each phase (max over ranks, mean over iterations after one warm-up); the byte
count is what the two all-to-alls move off rank 0.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    from ..config import ModelConfig
    from ..models.weights import _fp4_expert
    from ..ops import check_errors
    from ..ops import moe as moe_ops
    from ..parallel.comm import init_from_env
    from ..parallel.ep import EPMoE, local_expert_fn

    rank, world, local = init_from_env("nccl")
    dev = torch.device("cuda", local)
    cfg = ModelConfig()
    H, I, E, k, T = cfg.hidden_size, cfg.moe_intermediate, cfg.n_routed_experts, cfg.moe_topk, a.tokens
    ep = EPMoE(E)
    g = torch.Generator(device=dev).manual_seed(a.seed + 1000 * rank)
    w13, s13 = _fp4_expert(ep.local_experts, 2 * I, H, g, dev)
    w2, s2 = _fp4_expert(ep.local_experts, H, I, g, dev)
    lw = {"w13": w13, "s13": s13, "w2": w2, "s2": s2}
    moe_ops.prepare_experts_mx(lw, drop_canonical=False)
    shared_w13 = (torch.randn(2 * I, H, device=dev, generator=g) / H ** 0.5).bfloat16()
    shared_w2 = (torch.randn(H, I, device=dev, generator=g) / I ** 0.5).bfloat16()
    h = torch.randn(T, H, device=dev, generator=g).bfloat16()
    logits = torch.randn(T, E, device=dev, generator=g)
    top = logits.topk(k, dim=-1)
    ids, w = top.indices.int(), torch.softmax(top.values, -1)
    fn = local_expert_fn(lw, ep.expert_base, ep.local_experts, "mxfp4")
    phases = {"dispatch": [], "experts": [], "combine": [], "shared": [], "total": []}

    def event():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def shared_expert():
        x = h @ shared_w13.T
        return (torch.nn.functional.silu(x[:, :I]) * x[:, I:]) @ shared_w2.T

    multi = dist.is_initialized()
    total = None
    for it in range(a.iters + 1):
        if multi:
            dist.barrier()
        torch.cuda.synchronize(dev)
        box = {}

        def local(rows, lids):  # marks the end of the dispatch and of the expert compute
            box["d"] = event()
            y = fn(rows, lids)
            box["x"] = event()
            return y

        t0 = event()
        out = ep.forward(h, ids, w, local)
        t_comb = event()
        shared = shared_expert()
        t_sh = event()
        total = out + shared.float()
        t_end = event()
        torch.cuda.synchronize(dev)
        if it == 0:
            continue  # warm-up
        phases["dispatch"].append(t0.elapsed_time(box["d"]))
        phases["experts"].append(box["d"].elapsed_time(box["x"]))
        phases["combine"].append(box["x"].elapsed_time(t_comb))
        phases["shared"].append(t_comb.elapsed_time(t_sh))
        phases["total"].append(t0.elapsed_time(t_end))
    check_errors(dev)
    res = {}
    for key, vals in phases.items():
        t = torch.tensor([sum(vals) / len(vals)], dtype=torch.float64, device=dev)
        if multi:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[key + "_ms"] = round(float(t.item()), 3)
    sent = sum(c for r, c in enumerate(ep.last_counts["sent"]) if r != rank)
    if rank == 0:
        print(json.dumps({"case": "ep_moe_layer", "world": world, "tokens_per_rank": T, "experts": E, "topk": k,
                          "local_experts": ep.local_experts, "impl": "nccl all_to_all + packmla mxf4 experts",
                          **res, "tokens_per_s_per_rank": round(T / (res["total_ms"] / 1e3), 1),
                          "offrank_rows_sent_rank0": sent, "offrank_bytes_rank0": sent * H * 2 * 2,
                          "finite": bool(torch.isfinite(total).all())}), flush=True)
    if multi:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

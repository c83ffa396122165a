"""Launch the packmla server.

    python -m packmla.server --model tiny --device cpu --port 30000
    torchrun --nproc-per-node 4 -m packmla.server --model v4-flash --kv-cache-format direct --tp 4

Flags mirror the reference's launcher (scripts/local/run-server.sh:55-139): --kv-cache-format
native|direct, --tp, --mem-fraction-static, --max-running-requests, --context-length,
--chunked-prefill-size, --cuda-graph-bs, --disable-cuda-graph, --enable-hierarchical-cache,
--hicache-ratio, --moe-precision (the reference's flashinfer MXFP4 MoE precision option).
Rank 0 serves HTTP; the other ranks follow its schedule (packmla.server.driver).
"""
from __future__ import annotations

import argparse
import json
import os


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m packmla.server")
    ap.add_argument("--model", default="tiny", help="tiny | small | v4-flash | path to a packmla checkpoint")
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--kv-cache-format", default="direct", choices=["native", "direct"])
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--mem-fraction-static", type=float, default=0.88)
    ap.add_argument("--max-running-requests", type=int, default=64)
    ap.add_argument("--context-length", type=int, default=1 << 15)
    ap.add_argument("--chunked-prefill-size", type=int, default=8192)
    ap.add_argument("--cuda-graph-bs", type=int, nargs="*", default=None)
    ap.add_argument("--disable-cuda-graph", action="store_true")
    ap.add_argument("--enable-hierarchical-cache", action="store_true")
    ap.add_argument("--hicache-ratio", type=float, default=2.0)
    ap.add_argument("--moe-precision", default="default", choices=["default", "bf16"])
    ap.add_argument("--decode-impl", default="direct", choices=["direct", "adapter"])
    ap.add_argument("--collectives", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--seed", type=int, default=0)
    return ap


def model_config(name: str):
    from ..config import ModelConfig

    if name == "tiny":
        return ModelConfig.tiny(), None
    if name == "small":
        return ModelConfig(name="small", vocab_size=1000, hidden_size=1024, num_layers=4, num_heads=16,
                           q_lora_rank=256, o_groups=4, o_lora_rank=256, compress_ratios=[0, 4, 128, 4],
                           index_heads=8, index_topk=32, n_routed_experts=8, moe_topk=2, moe_intermediate=1024,
                           dense_format="bf16", max_position=1 << 16), None
    if name in ("v4-flash", "deepseek-v4-flash"):
        return ModelConfig(), None
    from ..models.weights import load_checkpoint

    W, cfg = load_checkpoint(name)
    return cfg, W


def build_engine(args, rank: int, local: int, world: int, comm):
    import torch

    from ..config import EngineConfig
    from ..engine.engine import Engine

    cfg, W = model_config(args.model)
    kw = {}
    if args.cuda_graph_bs:
        kw["cuda_graph_bs"] = args.cuda_graph_bs
    ecfg = EngineConfig(kv_cache_format=args.kv_cache_format, tp=world, ep=world,
                        mem_fraction_static=args.mem_fraction_static, max_running_requests=args.max_running_requests,
                        chunked_prefill_size=args.chunked_prefill_size, context_length=args.context_length,
                        disable_cuda_graph=args.disable_cuda_graph or args.device == "cpu",
                        enable_hierarchical_cache=args.enable_hierarchical_cache, hicache_ratio=args.hicache_ratio,
                        moe_precision=args.moe_precision, decode_impl=args.decode_impl, device=args.device,
                        random_seed=args.seed, **kw)
    dev = torch.device(args.device, local) if args.device == "cuda" else torch.device("cpu")
    if W is not None and dev.type == "cuda":
        W = {"layers": [{k: v.to(dev) for k, v in l.items()} for l in W["layers"]], "meta": W["meta"],
             **{k: v.to(dev) for k, v in W.items() if torch.is_tensor(v)}}
    kv_bytes = None if dev.type == "cuda" else 256 << 20
    eng = Engine.build(cfg, ecfg, dev, rank, world, comm, max_context=args.context_length,
                       max_requests=args.max_running_requests, kv_bytes=kv_bytes, seed=args.seed, weights=W)
    if dev.type == "cuda" and not ecfg.disable_cuda_graph:
        eng.runner.capture()
    return eng, ecfg


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    import torch
    import torch.distributed as dist

    from ..parallel.comm import TPComm, init_from_env
    from .driver import EngineDriver
    from .tokenizer import ByteTokenizer

    backend = "nccl" if args.device == "cuda" else "gloo"
    rank, world, local = init_from_env(backend)
    if world != args.tp:
        raise SystemExit(f"--tp {args.tp} but WORLD_SIZE={world}")
    cpu_group = dist.new_group(backend="gloo") if world > 1 else None
    comm = None
    if world > 1:
        if args.device == "cuda" and args.collectives == "fused":
            from ..parallel.fused import FusedComm

            comm = FusedComm(torch.device("cuda", local), model_config(args.model)[0].hidden_size)
        else:
            comm = TPComm()
    eng, ecfg = build_engine(args, rank, local, world, comm)
    driver = EngineDriver(eng, rank, world, cpu_group)
    name = args.served_model_name or os.path.basename(str(args.model))
    if rank != 0:
        driver.run_worker()
        return
    import uvicorn

    from .app import create_app

    app = create_app(driver, ByteTokenizer(eng.cfg.vocab_size), name, {"server_args": vars(args)})
    driver.start()
    print(json.dumps({"event": "server_ready", "host": args.host, "port": args.port,
                      "max_total_num_tokens": eng.capacity.max_total_tokens}), flush=True)
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="warning")
    finally:
        driver.stop()


if __name__ == "__main__":
    main()

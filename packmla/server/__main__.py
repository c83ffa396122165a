"""Launch the packmla server.

    python -m packmla.server --model tiny --device cpu --port 30000
    torchrun --nproc-per-node 4 -m packmla.server --model v4-flash --kv-cache-format direct --tp 4

Flags mirror the reference's launcher (scripts/local/run-server.sh:55-161): --kv-cache-format
native|direct, --tp, --mem-fraction-static, --max-running-requests, --context-length,
--chunked-prefill-size, --cuda-graph-bs, --disable-cuda-graph, --enable-hierarchical-cache,
--hicache-ratio, --moe-precision (the reference's flashinfer MXFP4 MoE precision option); the
reference's own flag names (--model-path, --random-seed, --cuda-graph-config, --kv-cache-dtype,
--moe-runner-backend, --ep, the --dsv4-c4-cache-* selectors, the HiCache policy flags, ...) are
accepted and mapped by `resolve_args`, so a reference launch line runs unchanged.
Rank 0 serves HTTP; the other ranks follow its schedule (packmla.server.driver).
"""
from __future__ import annotations

import argparse
import json
import os

from .reasoning import PARSERS as REASONING_PARSERS


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m packmla.server")
    ap.add_argument("--model", "--model-path", dest="model", default="tiny",
                    help="tiny | small | v4-flash | path to a packmla checkpoint")
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--api-key", default=None, help="require `Authorization: Bearer KEY` on every route but /health")
    ap.add_argument("--chat-preparation-workers", type=int, default=0, choices=[0, 1, 2, 4],
                    help="chat-template conversion on 1, 2 or 4 worker threads, admission bounded by the pool "
                         "(0: inline on the API loop; the reference's DSV4_ASYNC_PREPARATION / "
                         "DSV4_PREPARATION_WORKERS)")
    ap.add_argument("--frontend-diagnostics", action="store_true",
                    help="chat responses carry preparation and first-output stamps (FRONTEND_DIAGNOSTICS=1)")
    ap.add_argument("--tokenizer", "--tokenizer-path", dest="tokenizer", default=None,
                    help="directory with Hugging Face tokenizer files (local only); default: byte-level tokenizer")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--kv-cache-format", default="direct", choices=["native", "direct", "fp4-native", "fp4-direct"],
                    help="C4 cache: FP8 Native / Packed records, or the FP4 (V4.1) Native / Packed records")
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
    ap.add_argument("--seed", "--random-seed", dest="seed", type=int, default=0)
    ap.add_argument("--watchdog-timeout", type=float, default=1800.0,
                    help="seconds one engine step may take before /health reports the server unhealthy")
    ap.add_argument("--no-prefill-decode-interleave", action="store_true",
                    help="run waiting prefills before decode steps instead of alternating them")
    ap.add_argument("--max-total-tokens", type=int, default=None, help="cap the KV pool at this many tokens")
    # the reference launcher's flags (scripts/local/run-server.sh:55-161), mapped onto packmla's options
    ref = ap.add_argument_group("reference launcher flags")
    ref.add_argument("--kv-cache-dtype", default="fp8_e4m3", choices=["fp8_e4m3"],
                     help="C4 records are E4M3 + UE8M0 (the only supported cache dtype)")
    ref.add_argument("--cuda-graph-config", default=None,
                     help='JSON such as {"decode": {"backend": "full", "bs": [1, 2, 4]}, "prefill": {"backend": '
                          '"disabled"}}: decode graph batch sizes, or "disabled"')
    ref.add_argument("--moe-runner-backend", default="flashinfer_mxfp4", choices=["flashinfer_mxfp4"],
                     help="MXFP4 experts (packmla's tcgen05 MXFP4 x MXFP8 kernel)")
    ref.add_argument("--ep", "--ep-size", dest="ep", type=int, default=None,
                     help="expert-parallel size; packmla shards experts over the TP ranks, so it must equal --tp")
    ref.add_argument("--dsv4-c4-cache-format", default=None, choices=["native", "remnant"],
                     help="older selector: remnant = --kv-cache-format direct")
    ref.add_argument("--dsv4-c4-cache-implementation", default=None, choices=["kernel", "adapter"],
                     help="kernel = Direct Packed attention, adapter = Packed rows rebuilt as Native records")
    ref.add_argument("--dsv4-c4-cache-store-implementation", default="kernel", choices=["kernel"],
                     help="Packed records are written by the fused CUDA store kernel")
    ref.add_argument("--dsv4-c4-cache-keep-count", type=int, default=256)
    ref.add_argument("--dsv4-c4-cache-layer-keep-counts", default=None,
                     help="per-layer survivor counts: evaluation only (packmla.training.evaluate "
                          "--retention-sweep); serving accepts 256 for every layer")
    ref.add_argument("--hicache-io-backend", default="kernel", choices=["kernel", "direct"],
                     help="both move pages with packmla's segment-copy kernel")
    ref.add_argument("--hicache-mem-layout", default="page_first", choices=["page_first", "layer_first"],
                     help="host tier layout: all planes of a page together, or one region per plane")
    ref.add_argument("--hicache-write-policy", default="write_through", choices=["write_through"])
    ref.add_argument("--enable-metrics", action="store_true", help="accepted; /metrics is always served")
    ref.add_argument("--log-requests", action="store_true", help="log every finished request (JSON)")
    ref.add_argument("--log-requests-level", type=int, default=0, choices=[0, 1, 2, 3],
                     help="0 timing, 1 + sampling parameters, 2 + first 64 output ids, 3 + all token ids")
    ref.add_argument("--export-metrics-to-file", action="store_true",
                     help="append per-request metrics as JSON lines under --export-metrics-to-file-dir")
    ref.add_argument("--export-metrics-to-file-dir", default=None)
    ref.add_argument("--enable-dp-attention", action="store_true",
                     help="each rank serves its own requests with every attention head; routed experts stay "
                          "split, MoE tokens are exchanged between the ranks (NCCL)")
    ref.add_argument("--disable-radix-cache", action="store_true",
                     help="release a finished request's KV at once instead of keeping it on the device for a "
                          "later prompt that extends it")
    for flag in ("--skip-server-warmup", "--trust-remote-code", "--disable-overlap-schedule",
                 "--disable-flashinfer-autotune", "--language-model-only"):
        ref.add_argument(flag, action="store_true", help="accepted; no effect in packmla")
    ref.add_argument("--reasoning-parser", default=None, choices=sorted(REASONING_PARSERS),
                     help="chat messages carry the output's think block as reasoning_content")
    for flag in ("--tool-call-parser", "--model-type", "--dsa-decode-backend",
                 "--dsa-prefill-backend", "--dsv4-attn-backend"):
        ref.add_argument(flag, default=None, help="accepted; no effect in packmla")
    return ap


def resolve_args(args) -> dict:
    """EngineConfig settings of the parsed flags (reference flags folded in); raises SystemExit on a
    combination packmla does not serve."""
    fmt = args.kv_cache_format
    if args.dsv4_c4_cache_format is not None:
        fmt = "direct" if args.dsv4_c4_cache_format == "remnant" else "native"
    impl = args.decode_impl
    if args.dsv4_c4_cache_implementation is not None:
        impl = "adapter" if args.dsv4_c4_cache_implementation == "adapter" else "direct"
    if args.ep is not None and args.ep != args.tp:
        raise SystemExit(f"--ep {args.ep}: packmla shards the routed experts over the TP ranks (EP = TP = {args.tp})")
    layer_counts = None
    if args.dsv4_c4_cache_layer_keep_counts:  # "layer:count,layer:count" (model layer indices of C4 layers)
        layer_counts = {}
        for item in args.dsv4_c4_cache_layer_keep_counts.replace(" ", "").split(","):
            if item:
                layer, count = item.split(":")
                layer_counts[int(layer)] = int(count)
    kw = dict(kv_cache_format=fmt, decode_impl=impl, keep_count=args.dsv4_c4_cache_keep_count,
              layer_keep_counts=layer_counts,
              prefill_decode_interleave=not args.no_prefill_decode_interleave,
              prefix_cache=not args.disable_radix_cache, hicache_mem_layout=args.hicache_mem_layout,
              dp_attention=bool(getattr(args, "enable_dp_attention", False)) and args.tp > 1)
    disable_graphs = args.disable_cuda_graph or args.device == "cpu"
    bs = args.cuda_graph_bs
    if args.cuda_graph_config:
        gc = json.loads(args.cuda_graph_config)
        dec = gc.get("decode", {})
        if dec.get("backend", "full") == "disabled":
            disable_graphs = True
        elif dec.get("bs"):
            bs = [int(b) for b in dec["bs"]]
    if bs:
        kw["cuda_graph_bs"] = bs
    kw["disable_cuda_graph"] = disable_graphs
    return kw


def request_logger(args):
    """The `RequestLogger` of the --log-requests / --export-metrics-to-file flags (None when both are off)."""
    from .request_log import RequestLogger

    if args.export_metrics_to_file and not args.export_metrics_to_file_dir:
        raise SystemExit("--export-metrics-to-file needs --export-metrics-to-file-dir")
    export = args.export_metrics_to_file_dir if args.export_metrics_to_file else None
    if not args.log_requests and export is None:
        return None
    if args.log_requests:
        import logging

        logging.basicConfig(level=logging.INFO, format="%(asctime)s %(name)s %(message)s")
    return RequestLogger(args.log_requests, args.log_requests_level, export)


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
    ecfg = EngineConfig(tp=world, ep=world, mem_fraction_static=args.mem_fraction_static,
                        max_running_requests=args.max_running_requests,
                        chunked_prefill_size=args.chunked_prefill_size, context_length=args.context_length,
                        enable_hierarchical_cache=args.enable_hierarchical_cache, hicache_ratio=args.hicache_ratio,
                        moe_precision=args.moe_precision, device=args.device, random_seed=args.seed,
                        **resolve_args(args))
    try:
        ecfg.validate()
    except ValueError as exc:
        raise SystemExit(f"unsupported configuration: {exc}") from exc
    dev = torch.device(args.device, local) if args.device == "cuda" else torch.device("cpu")
    if W is not None and dev.type == "cuda":
        W = {"layers": [{k: v.to(dev) for k, v in l.items()} for l in W["layers"]], "meta": W["meta"],
             **{k: v.to(dev) for k, v in W.items() if torch.is_tensor(v)}}
    kv_bytes = None if dev.type == "cuda" else 256 << 20
    if args.max_total_tokens:
        from ..kv.pool import bytes_per_full_token, fixed_bytes

        kv_bytes = int(args.max_total_tokens * bytes_per_full_token(cfg, ecfg.kv_cache_format,
                                                                    ecfg.swa_full_tokens_ratio, ecfg.keep_for)
                       + fixed_bytes(cfg, args.max_running_requests + 1))
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
    from .tokenizer import load_tokenizer

    backend = "nccl" if args.device == "cuda" else "gloo"
    rank, world, local = init_from_env(backend)
    if world != args.tp:
        raise SystemExit(f"--tp {args.tp} but WORLD_SIZE={world}")
    cpu_group = dist.new_group(backend="gloo") if world > 1 else None
    comm = None
    if world > 1:
        if args.device == "cuda" and args.collectives == "fused" and not args.enable_dp_attention:
            from ..parallel.fused import FusedComm

            comm = FusedComm(torch.device("cuda", local), model_config(args.model)[0].hidden_size)
        else:
            comm = TPComm()
    eng, ecfg = build_engine(args, rank, local, world, comm)
    driver = EngineDriver(eng, rank, world, cpu_group, watchdog_s=args.watchdog_timeout,
                          request_logger=request_logger(args) if rank == 0 else None)
    name = args.served_model_name or os.path.basename(str(args.model))
    if rank != 0:
        driver.run_worker()
        return
    import uvicorn

    from .app import create_app

    app = create_app(driver, load_tokenizer(args.tokenizer, eng.cfg.vocab_size), name,
                     {"server_args": {k: v for k, v in vars(args).items() if k != "api_key"}}, api_key=args.api_key,
                     preparation_workers=args.chat_preparation_workers,
                     frontend_diagnostics=args.frontend_diagnostics, reasoning_parser=args.reasoning_parser)
    driver.start()
    print(json.dumps({"event": "server_ready", "host": args.host, "port": args.port,
                      "max_total_num_tokens": eng.capacity.max_total_tokens}), flush=True)
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="warning")
    finally:
        driver.stop()


if __name__ == "__main__":
    main()

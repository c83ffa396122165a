"""Model-free kernel microbenchmarks (device time with CUDA events, L2 flushed between runs).

    python -m packmla.bench.microbench moe   [--tokens 40] [--experts 256] [--topk 8]
    python -m packmla.bench.microbench decode [--batch 16] [--heads 128] [--context 32768] [--topk 2048]
    python -m packmla.bench.microbench store  [--rows 24]
    python -m packmla.bench.microbench decode-paired [--batch 16] [--context 32768] [--with-adapter]
    python -m packmla.bench.microbench decode-suite [--paired] > suite.jsonl
    python -m packmla.bench.microbench judge --results suite.jsonl [--paired] [--rounds 30]
    python -m packmla.bench.microbench glm-suite [--rounds 30] [--glm-batches 1,8,16,24] [--out F [--resume]]

Each case prints one JSON line: mean microseconds, achieved bytes/s and the fraction of the
measured HBM copy bandwidth (MEASURED_PEAKS.json, "of measured").

Reference protocol: 30 rounds after 10 warm-ups, CUDA-graph-free device timing of the
operation only (benchmarks/microbench/dsv4-flash-decode-store/README.md:11-23).  Paired rounds
(`decode-paired`, `decode-suite --paired`; reference: the balanced paired timing loop of its
GLM/V4.1 suites) time every mode once per round, in an order rotated each round so drift and
position effects cancel, and report each mode's mean and the per-round latency ratios against the
first mode (geometric mean, min, max).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def measured_hbm_gbs() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "of measured"
    return 6650.0, "of fallback"


class L2Flush:
    def __init__(self, device, nbytes: int = 256 << 20):
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)

    def __call__(self):
        self.buf.fill_(1)


LAST_CLOCKS: dict = {}


def time_op(fn, rounds: int, warmup: int, device, flush: L2Flush | None, graph: bool = False) -> float:
    """Mean microseconds over `rounds` (each round timed alone, L2 flushed before it).

    graph=True captures fn once in a CUDA graph and times its replays, so the host-side launch work
    (argument checks, tensor-map encoding) stays out of the measurement, as in the engine's decode graphs.
    """
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        fn = g.replay
        fn()
        torch.cuda.synchronize(device)
    from .timing import ClockSampler

    total = 0.0
    # timed rounds first; then more untimed rounds until the 200 ms clock sampler has seen the work
    with ClockSampler(torch.device(device).index or 0) as clk:
        t_end = time.perf_counter() + 0.8
        n = 0
        while n < rounds or time.perf_counter() < t_end:
            if flush is not None:
                flush()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize(device)
            if n < rounds:
                total += s.elapsed_time(e)
            n += 1
    LAST_CLOCKS.clear()
    LAST_CLOCKS.update(clk.summary())
    return total / rounds * 1e3


def time_op_replays(fn, rounds: int, warmup: int, device, replays: int = 100) -> float:
    """The reference's decode timing protocol: one CUDA graph of `replays` back-to-back calls per sample,
    no cache flush; mean microseconds per call over `rounds` samples."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(replays):
            fn()
    g.replay()
    torch.cuda.synchronize(device)
    from .timing import ClockSampler

    total = 0.0
    with ClockSampler(torch.device(device).index or 0) as clk:
        t_end = time.perf_counter() + 0.8
        n = 0
        while n < rounds or time.perf_counter() < t_end:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            g.replay()
            e.record()
            torch.cuda.synchronize(device)
            if n < rounds:
                total += s.elapsed_time(e)
            n += 1
    LAST_CLOCKS.clear()
    LAST_CLOCKS.update(clk.summary())
    return total / rounds / replays * 1e3


def bench_moe(args, dev):
    from packmla.config import ModelConfig
    from packmla.models.weights import _fp4_expert
    from packmla.ops import check_errors
    from packmla.ops import moe as moe_ops

    cfg = ModelConfig()
    H, I, E, k = cfg.hidden_size, cfg.moe_intermediate, args.experts, args.topk
    g = torch.Generator(device=dev).manual_seed(0)
    lw = {}
    lw["w13"], lw["s13"] = _fp4_expert(E, 2 * I, H, g, dev)
    lw["w2"], lw["s2"] = _fp4_expert(E, H, I, g, dev)
    if args.precision == "bf16":
        moe_ops.prepare_experts(lw)
    else:
        moe_ops.prepare_experts_mx(lw)
    h = torch.randn(args.tokens, H, device=dev, generator=g).bfloat16()
    gate = torch.randn(E, H, device=dev, generator=g).bfloat16() * H ** -0.5
    ids, w = moe_ops.route(h, gate, torch.zeros(E, device=dev), k, 1.0)
    active = int(torch.unique(ids).numel())
    fn = lambda: moe_ops.experts(h, ids, w, lw, 0, E, "mxfp4", precision=args.precision)  # noqa: E731
    us = time_op(fn, args.rounds, args.warmup, dev, L2Flush(dev), graph=True)
    check_errors(dev)
    waits = None
    if args.precision == "default" and args.prof:
        prof = torch.zeros(16, dtype=torch.int64, device=dev)
        moe_ops.experts(h, ids, w, lw, 0, E, "mxfp4", precision="default", prof=prof)
        torch.cuda.synchronize(dev)
        pv = prof.tolist()
        names = ["producer_wait_stage", "mma_wait_data", "mma_wait_accum", "epilogue_wait_accum", "producer_life",
                 "mma_wait_scales", "mma_issue", "producer_issue"]
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        waits = {f"{tag}_{n}_kcycles_per_cta": round(pv[o + i] / 1e3 / sms, 1)
                 for o, tag in ((0, "gateup"), (8, "down")) for i, n in enumerate(names)}
    per_expert = (2 * I * H + H * I) // 2 + (2 * I * H + H * I) // 32
    nbytes = active * per_expert
    peak, tag = measured_hbm_gbs()
    gbs = nbytes / us / 1e3
    flops = 2 * args.tokens * k * 3 * H * I  # gate, up and down GEMMs of every routed (token, expert) pair
    return {"case": "moe_fp4", "precision": args.precision, "waits": waits, "tokens": args.tokens, "experts": E, "topk": k, "active_experts": active,
            "us": round(us, 2), "TFLOPs": round(flops / us / 1e6, 1), "weight_bytes": nbytes, "GBps": round(gbs, 1),
            "hbm_fraction": round(gbs / peak, 3), "peak_note": tag}


def bench_decode(args, dev):
    from packmla.formats import abi, codec
    from packmla.ops import attention as attn_ops
    from packmla.ops import check_errors
    from packmla.ops import kv as kv_ops

    B, Hh, K, W = args.batch, args.heads, args.topk, args.swa
    records = args.context // abi.C4_RATIO
    g = torch.Generator(device=dev).manual_seed(0)
    freqs = kv_ops.freq_table_f32(codec.rope_table(args.context + 1024)).to(dev)
    w = torch.ones(512, device=dev)
    rows = B * records  # each query owns its own context
    swa_rows = max(1, B * W)
    swa_pool = torch.zeros(((swa_rows + 63) // 64) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
    kv_ops.native_store(torch.randn(swa_rows, 512, device=dev, generator=g), w, 1e-6,
                        torch.arange(swa_rows, device=dev), torch.arange(swa_rows, device=dev) % args.context, freqs,
                        swa_pool)
    planes, pool = None, None
    chunk = 1 << 18
    if args.kv_format in ("direct", "adapter"):
        planes = attn_ops.PackedPlanes(torch.zeros(rows, 256, dtype=torch.uint8, device=dev),
                                       torch.zeros(rows, 8, dtype=torch.int64, device=dev),
                                       torch.zeros(rows, 8, dtype=torch.uint8, device=dev))
        for a in range(0, rows, chunk):
            b = min(rows, a + chunk)
            kv_ops.packed_store(torch.randn(b - a, 512, device=dev, generator=g), w, 1e-6,
                                torch.arange(a, b, device=dev), planes.values, planes.bitmap, planes.scales)
        rec_bytes = abi.PACKED_RECORD_BYTES
    elif args.kv_format.startswith("fp4-"):
        from packmla.formats import fp4

        fmt4 = args.kv_format[4:]
        pool = torch.zeros(((rows + 63) // 64) * fp4.page_bytes(fmt4), dtype=torch.uint8, device=dev)
        for a in range(0, rows, chunk):
            b = min(rows, a + chunk)
            kv_ops.fp4_store(torch.randn(b - a, 512, device=dev, generator=g), w, 1e-6,
                             torch.arange(a, b, device=dev), (torch.arange(a, b, device=dev) % records) * 4,
                             freqs, pool, fmt4 == "direct")
        rec_bytes = fp4.record_bytes(fmt4)
    else:
        pool = torch.zeros(((rows + 63) // 64) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
        for a in range(0, rows, chunk):
            b = min(rows, a + chunk)
            kv_ops.native_store(torch.randn(b - a, 512, device=dev, generator=g), w, 1e-6,
                                torch.arange(a, b, device=dev), (torch.arange(a, b, device=dev) % records) * 4,
                                freqs, pool)
        rec_bytes = abi.NATIVE_RECORD_BYTES
    base = (torch.arange(B, device=dev) * records)[:, None]
    sel = torch.stack([torch.randperm(records, device=dev, generator=g)[:K] for _ in range(B)])
    csa_slots = (base + sel).int().contiguous()
    csa_pos = (sel * 4).int().contiguous()
    swa_slots = (torch.arange(B, device=dev)[:, None] * W + torch.arange(max(W, 1), device=dev)[None]).int()
    q = (torch.randn(B, Hh, 512, device=dev, generator=g) / 2).bfloat16()
    args_d = dict(swa_slots=swa_slots, swa_len=torch.full((B,), W, dtype=torch.int32, device=dev),
                  csa_slots=csa_slots, csa_pos=csa_pos, csa_len=torch.full((B,), K, dtype=torch.int32, device=dev),
                  freqs=freqs, sink=torch.zeros(Hh, device=dev), scale=512 ** -0.5,
                  q_pos=torch.full((B,), args.context - 1, dtype=torch.int32, device=dev), csa_pool=pool,
                  csa_planes=planes)
    if args.kv_format.startswith("fp4-"):
        args_d["csa_fp4"] = args.kv_format[4:]
    splits = args.splits or attn_ops.choose_splits(B, Hh, max(W, 1) + K, max_clusters=attn_ops.max_active_clusters(dev))
    ws = attn_ops.DecodeWorkspace(B, Hh, splits, dev)
    out = torch.empty(B, Hh, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, Hh, dtype=torch.float32, device=dev)
    fn = lambda: attn_ops.sparse_mla_decode(q, swa_pool, workspace=ws, out=out, lse=lse, **args_d)  # noqa: E731
    if args.kv_format == "adapter":
        # reference "Adapter" mode: reconstruct the selected Packed rows into a Native workspace, then the
        # Native decode reads the workspace
        n = B * K
        wsn = torch.zeros(((n + 63) // 64) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
        dst = torch.arange(n, device=dev, dtype=torch.int64)
        src_rows, src_pos = csa_slots.reshape(-1).contiguous(), csa_pos.reshape(-1).contiguous()
        args_a = dict(args_d, csa_pool=wsn, csa_planes=None,
                      csa_slots=dst.view(B, K).int().contiguous())

        def fn():
            kv_ops.packed_to_native(planes.values, planes.bitmap, planes.scales, src_rows, src_pos, freqs, wsn, dst)
            return attn_ops.sparse_mla_decode(q, swa_pool, workspace=ws, out=out, lse=lse, **args_a)
    nbytes = B * (K * rec_bytes + W * abi.NATIVE_RECORD_BYTES) + q.numel() * 2 + out.numel() * 2
    if getattr(args, "build_only", False):
        return fn, {"kv_format": args.kv_format, "bytes": nbytes, "splits": ws.splits}
    if args.protocol == "reference":
        us = time_op_replays(fn, args.rounds, args.warmup, dev)
    else:
        us = time_op(fn, args.rounds, args.warmup, dev, L2Flush(dev), graph=True)
    check_errors(dev)
    stamps = None
    if args.prof and args.kv_format != "adapter":
        prof = torch.zeros(64, dtype=torch.int64, device=dev)
        prof[59] = 2 ** 63 - 1  # earliest CTA start (atomic min)
        prof[46] = 2 ** 63 - 1  # earliest staged epilogue (atomic min)
        if args.protocol != "reference":  # the reference protocol's stamps come from a warm run
            L2Flush(dev)()
        attn_ops.sparse_mla_decode(q, swa_pool, workspace=ws, out=out, lse=lse, prof=prof, **args_d)
        torch.cuda.synchronize(dev)
        pv = prof.tolist()
        t0 = pv[0]
        names = ["setup"] + [f"{k}{i}" for i in range(8) for k in ("E", "X")]  # per tile: expanded, softmaxed
        stamps = {n: round((pv[1 + i] - t0) / 1e3, 2) for i, n in enumerate(names) if pv[1 + i]}
        stamps.update({f"S{i}": round((pv[18 + i] - t0) / 1e3, 2) for i in range(8) if pv[18 + i]})
        stamps.update({f"PV{i}": round((pv[26 + i] - t0) / 1e3, 2) for i in range(8) if pv[26 + i]})
        stamps.update({f"X0.{n}": round((pv[36 + i] - t0) / 1e3, 2) for i, n in
                       enumerate(["start", "scores", "maxima", "probs", "m_updated", "p_computed"]) if pv[36 + i]})
        stamps.update({"epilogue": round((pv[34] - t0) / 1e3, 2), "end": round((pv[35] - t0) / 1e3, 2),
                       "unit": "us after the start of the last split of query 0, head group 0"})
        extra = {44: "L1.fetched", 48: "ep.stats", 49: "ep.tmem_ld", 45: "cl.weights", 50: "ep.staged", 51: "ep.written", 52: "cl.ready", 53: "cl.received",
                 54: "su.load0", 55: "su.idx1", 56: "su.q_converted"}
        stamps.update({n: round((pv[i] - t0) / 1e3, 2) for i, n in extra.items() if pv[i]})
        stamps.update({"cta_first_start": round((pv[59] - t0) / 1e3, 2),
                       "cta_last_start": round((pv[58] - t0) / 1e3, 2),
                       "cta_last_end": round((pv[57] - t0) / 1e3, 2)})
        if pv[47]:
            stamps.update({"cta_first_staged": round((pv[46] - t0) / 1e3, 2),
                           "cta_last_staged": round((pv[47] - t0) / 1e3, 2)})
    flops = 4 * B * Hh * (K + W) * 512
    peak, tag = measured_hbm_gbs()
    gbs = nbytes / us / 1e3
    return {"case": "sparse_mla_decode", "rounds": args.rounds, "protocol": args.protocol, "stamps": stamps,
            "kv_format": args.kv_format,
            "batch": B,
            "heads": Hh, "topk": K,
            "swa": W, "context": args.context, "splits": ws.splits, "tile_rows": attn_ops.TILE_ROWS, "us": round(us, 2), "bytes": nbytes,
            "GBps": round(gbs, 1), "hbm_fraction": round(gbs / peak, 3), "TFLOPs": round(flops / us / 1e6, 1),
            "peak_note": tag}


def paired_rounds(timers: dict, rounds: int) -> dict:
    """Run every timer once per round, the order rotated by one mode each round; timers return
    microseconds.  Ratios are per round against the first mode."""
    modes = list(timers)
    if rounds < 1 or not modes:
        raise ValueError("at least one round and one mode required")
    samples = {m: [] for m in modes}
    for r in range(rounds):
        k = r % len(modes)
        for m in modes[k:] + modes[:k]:
            samples[m].append(float(timers[m]()))
    base = modes[0]
    out = {"rounds": rounds, "order": "rotated", "baseline": base,
           "mean_us": {m: round(sum(v) / len(v), 3) for m, v in samples.items()}, "ratio": {}}
    for m in modes[1:]:
        ratios = [a / b for a, b in zip(samples[m], samples[base])]
        geo = math.exp(sum(math.log(x) for x in ratios) / len(ratios))
        out["ratio"][f"{m}/{base}"] = {"geomean": round(geo, 5), "change_pct": round((geo - 1) * 100, 3),
                                       "min": round(min(ratios), 5), "max": round(max(ratios), 5)}
    return out


def bench_decode_paired(args, dev, modes=("native", "direct")) -> dict:
    """Decode modes built side by side, each captured in a CUDA graph, timed in paired rounds."""
    import copy

    from packmla.ops import check_errors

    from .timing import ClockSampler

    flush = L2Flush(dev)
    graphs, meta = {}, {}
    for m in modes:
        a = copy.copy(args)
        a.kv_format, a.build_only = m, True
        fn, meta[m] = bench_decode(a, dev)
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        graphs[m] = g
    check_errors(dev)

    def timer(g):
        def run() -> float:
            flush()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            g.replay()
            e.record()
            torch.cuda.synchronize(dev)
            return s.elapsed_time(e) * 1e3
        return run

    with ClockSampler(torch.device(dev).index or 0) as clk:
        res = paired_rounds({m: timer(graphs[m]) for m in modes}, args.rounds)
    check_errors(dev)
    for g in graphs.values():
        g.reset()
    return {"case": "sparse_mla_decode_paired", "batch": args.batch, "heads": args.heads, "topk": args.topk,
            "swa": args.swa, "context": args.context, "modes": meta, **res, "clocks": clk.summary()}


# the reference's table also has batches 32 and 64; the device GLM decode is limited to batch 24
# (packmla.ops.glm.MAX_DEVICE_BATCH)
GLM_SUITE_BATCHES, GLM_SUITE_TAILS, GLM_SUITE_CACHES = (1, 8, 16, 24), (0, 3), ("warm", "rotating")


def bench_glm(args, dev) -> list[dict]:
    """GLM-5.3 decode, Native (512 B rows) vs Direct (320 B Packed rows): the reference's upstream-decode
    protocol shape (benchmarks/microbench/glm53-flash-packed/README.md:1-40): 16 local heads (TP4), one
    query per sequence selecting top-k 2048 rows plus 0 or 3 tail rows of a 131076-token context, batches
    1 .. 24 (the reference's 32 and 64 exceed the device limit of `packmla.ops.glm`); "warm" reuses one input bank (L2-resident), "rotating" flushes L2 before every sample.  Both
    modes are CUDA graphs timed in paired rounds; one JSON row per case."""
    from packmla.formats import glm
    from packmla.ops import check_errors
    from packmla.ops.attention import DecodeWorkspace, choose_splits, max_active_clusters
    from packmla.ops.glm import MAX_DEVICE_BATCH, GLMPlanes, glm_sparse_decode, glm_store

    if max(args.glm_batches) > MAX_DEVICE_BATCH:
        raise SystemExit(f"glm-suite: batches above {MAX_DEVICE_BATCH} stay off the device")

    from .timing import ClockSampler

    ctx, H = args.context, args.heads
    rec = None
    if getattr(args, "out", None):
        from .suite_record import SuiteRecord

        rec = SuiteRecord(args.out, {"suite": "glm", "seed": 20261024, "context": ctx, "heads": H,
                                     "rounds": args.rounds, "warmup": args.warmup}, resume=args.resume)
    g = torch.Generator(device=dev).manual_seed(20261024)
    pool = torch.empty(ctx, 512, dtype=torch.uint8, device=dev)
    planes = GLMPlanes(torch.empty(ctx, 256, dtype=torch.uint8, device=dev),
                       torch.empty(ctx, 8, dtype=torch.int64, device=dev))
    w = torch.rand(512, device=dev, generator=g) + 0.5
    for s0 in range(0, ctx, 1 << 16):
        n = min(1 << 16, ctx - s0)
        raw = torch.randn(n, 512, device=dev, generator=g)
        slots = torch.arange(s0, s0 + n, device=dev)
        glm_store(raw, w, 1e-6, slots, pool=pool)
        glm_store(raw, w, 1e-6, slots, planes=planes)
    check_errors(dev)
    flush = L2Flush(dev)
    rows_out = []
    for batch in args.glm_batches:
        for tails in GLM_SUITE_TAILS:
            names = {c: f"glm_decode_h{H}_q1_t{tails}_b{batch}_{c}" for c in GLM_SUITE_CACHES}
            if rec is not None and all(n in rec.done for n in names.values()):
                continue  # measured by the run being resumed
            K = glm.GLM53.index_topk + tails
            q = torch.randn(batch, H, 512, device=dev, generator=g).bfloat16()
            sel = torch.stack([torch.randperm(ctx - tails, device=dev, generator=g)[:glm.GLM53.index_topk]
                               for _ in range(batch)]).int()
            if tails:
                tail = torch.arange(ctx - tails, ctx, device=dev, dtype=torch.int32).expand(batch, tails)
                sel = torch.cat((sel, tail), 1)
            sel = sel.contiguous()
            lens = torch.full((batch,), K, dtype=torch.int32, device=dev)
            ws = DecodeWorkspace(batch, H, choose_splits(batch, H, K, max_clusters=max_active_clusters(dev)), dev)
            graphs = {}
            for mode, kw in (("native", {"pool": pool}), ("direct", {"planes": planes})):
                out = torch.empty(batch, H, 512, dtype=torch.bfloat16, device=dev)
                lse = torch.empty(batch, H, dtype=torch.float32, device=dev)
                fn = (lambda kw=kw, out=out, lse=lse:
                      glm_sparse_decode(q, sel, lens, workspace=ws, out=out, lse=lse, **kw))
                for _ in range(args.warmup):
                    fn()
                torch.cuda.synchronize(dev)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    fn()
                graphs[mode] = gr
            check_errors(dev)
            for cache in GLM_SUITE_CACHES:
                if rec is not None and names[cache] in rec.done:
                    continue

                def timer(gr, cold=cache == "rotating"):
                    def run() -> float:
                        if cold:
                            flush()
                        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        s.record()
                        gr.replay()
                        e.record()
                        torch.cuda.synchronize(dev)
                        return s.elapsed_time(e) * 1e3
                    return run

                with ClockSampler(torch.device(dev).index or 0) as clk:
                    t_end = time.perf_counter() + 0.8
                    res = paired_rounds({m: timer(gr) for m, gr in graphs.items()}, args.rounds)
                    while time.perf_counter() < t_end:  # untimed replays until the sampler has seen the work
                        for gr in graphs.values():
                            gr.replay()
                        torch.cuda.synchronize(dev)
                row = {"case": names[cache], "batch": batch, "heads": H,
                       "rows_per_query": K, "context": ctx, "splits": ws.splits, **res, "clocks": clk.summary()}
                print(json.dumps(row), flush=True)
                if rec is not None:
                    rec.write(row)
                rows_out.append(row)
            for gr in graphs.values():
                gr.reset()
    check_errors(dev)
    return rows_out


SUITE_CONTEXTS, SUITE_BATCHES, SUITE_FORMATS = (32768, 131072), (1, 16, 64), ("native", "direct")
FP4_SUITE_BATCHES = (8, 16, 24, 28, 32)
BAD_CLOCK_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def judge(rows: list[dict], rounds: int, paired: bool = False, min_clock_fraction: float = 0.8) -> dict:
    """Accept or reject a decode-suite run: every case of the grid present once, each timed over
    `rounds` rounds with finite positive times, and a clock record without hardware or thermal
    slowdown and not stuck below `min_clock_fraction` of the maximum with no reason given (a leftover
    clock lock).  `sw_power_cap` is accepted and noted.  Returns the verdict with its reasons."""
    key = (lambda r: (r["context"], r["batch"])) if paired else (lambda r: (r["context"], r["batch"], r["kv_format"]))
    expected = ({(c, b) for c in SUITE_CONTEXTS for b in SUITE_BATCHES} if paired else
                {(c, b, f) for c in SUITE_CONTEXTS for b in SUITE_BATCHES for f in SUITE_FORMATS})
    seen: dict = {}
    rejected, notes = [], []
    for r in rows:
        k = key(r)
        if k in seen:
            rejected.append({"case": list(k), "reason": "duplicate case"})
        seen[k] = r
        times = list(r["mean_us"].values()) if paired else [r.get("us")]
        if r.get("rounds") != rounds:
            rejected.append({"case": list(k), "reason": f"rounds {r.get('rounds')} != {rounds}"})
        if any(t is None or not math.isfinite(t) or t <= 0 for t in times):
            rejected.append({"case": list(k), "reason": "non-finite or non-positive time"})
        clk = r.get("clocks") or {}
        reasons = clk.get("reasons") or []
        bad = [x for x in reasons if x in BAD_CLOCK_REASONS]
        if bad:
            rejected.append({"case": list(k), "reason": "clock slowdown: " + ", ".join(bad)})
        elif "unavailable" in reasons or not clk.get("sm_mhz") or not clk.get("sm_max_mhz"):
            rejected.append({"case": list(k), "reason": "no clock record"})
        elif clk["sm_mhz"] < min_clock_fraction * clk["sm_max_mhz"] and "sw_power_cap" not in reasons:
            rejected.append({"case": list(k), "reason": f"SM clock {clk['sm_mhz']} MHz well below max with no reason"})
        if "sw_power_cap" in reasons:
            notes.append({"case": list(k), "note": "sw_power_cap active"})
    missing = sorted(list(k) for k in expected - set(seen))
    return {"passed": not missing and not rejected, "cases": len(seen), "expected": len(expected),
            "missing": missing, "rejected": rejected, "notes": notes}


def bench_store(args, dev):
    from packmla.formats import abi, codec
    from packmla.ops import kv as kv_ops

    R = args.rows
    g = torch.Generator(device=dev).manual_seed(0)
    raw = torch.randn(R, 512, device=dev, generator=g)
    w = torch.ones(512, device=dev)
    slots = torch.randperm(R * 4, device=dev, generator=g)[:R]
    freqs = kv_ops.freq_table_f32(codec.rope_table(1 << 16)).to(dev)
    pos = torch.randint(0, 1 << 16, (R,), device=dev, generator=g)
    pool = torch.zeros(((4 * R + 63) // 64) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
    v = torch.zeros(4 * R, 256, dtype=torch.uint8, device=dev)
    bm = torch.zeros(4 * R, 8, dtype=torch.int64, device=dev)
    sc = torch.zeros(4 * R, 8, dtype=torch.uint8, device=dev)
    fn_n = lambda: kv_ops.native_store(raw, w, 1e-6, slots, pos, freqs, pool)  # noqa: E731
    fn_p = lambda: kv_ops.packed_store(raw, w, 1e-6, slots, v, bm, sc)  # noqa: E731
    if args.protocol == "reference":
        native = time_op_replays(fn_n, args.rounds, args.warmup, dev)
        packed = time_op_replays(fn_p, args.rounds, args.warmup, dev)
    else:
        native = time_op(fn_n, args.rounds, args.warmup, dev, None)
        packed = time_op(fn_p, args.rounds, args.warmup, dev, None)
    return {"case": "kv_store", "rows": R, "protocol": args.protocol, "native_us": round(native, 3),
            "packed_us": round(packed, 3)}


def bench_index(args, dev):
    """Indexer of one C4 layer: B queries x 64 heads x 128 over the `context` / 4 records of each query's
    request (FP8 keys), logits + top-k (csrc/indexer.cu), V4-Flash shapes."""
    from packmla.config import ModelConfig
    from packmla.ops import indexer as idx_ops

    cfg = ModelConfig()
    B, R = args.batch, args.context // 4
    K = args.topk or cfg.index_topk
    g = torch.Generator(device=dev).manual_seed(0)
    keys = torch.zeros(B * R, 128, dtype=torch.uint8, device=dev)
    scales = torch.zeros(B * R, dtype=torch.float32, device=dev)
    idx_ops.index_key_store(torch.randn(B * R, 128, device=dev, generator=g), torch.arange(B * R, device=dev),
                            keys, scales)
    phys = (torch.arange(B, device=dev)[:, None] * R + torch.arange(R, device=dev)[None]).int().contiguous()
    count = torch.full((B,), R, dtype=torch.int64, device=dev)
    q = torch.randn(B, cfg.index_heads, cfg.index_dim, device=dev, generator=g).bfloat16()
    w = torch.rand(B, cfg.index_heads, device=dev, generator=g)
    fn = lambda: idx_ops.index_select(q, w, keys, scales, phys, count, R, K)  # noqa: E731
    if args.protocol == "reference":
        us = time_op_replays(fn, args.rounds, args.warmup, dev)
    else:
        us = time_op(fn, args.rounds, args.warmup, dev, L2Flush(dev), graph=True)
    nbytes = B * R * (128 + 4 + 4) + B * cfg.index_heads * cfg.index_dim * 2 + B * K * 8
    peak, tag = measured_hbm_gbs()
    gbs = nbytes / us / 1e3
    flops = 2 * B * R * cfg.index_heads * cfg.index_dim
    return {"case": "index_select", "protocol": args.protocol, "batch": B, "context": args.context, "records": R,
            "topk": K, "heads": cfg.index_heads, "us": round(us, 2), "bytes": nbytes, "GBps": round(gbs, 1),
            "hbm_fraction": round(gbs / peak, 3), "fp8_TFLOPs": round(flops / us / 1e6, 1), "peak_note": tag}


# V4-Flash decode projections (N, K, batch) at TP = 1: fused attention input, q up-projection + indexer
# query, grouped output LoRA, output projection, shared expert + gate, shared down, LM head
DENSE_SHAPES = {"w_h": (3904, 4096, 1), "wq_b+wi_q": (40960, 1024, 1), "wo_a": (1024, 4096, 8),
                "wo_b": (4096, 8192, 1), "w_ffn": (4352, 4096, 1), "shared_w2": (4096, 2048, 1),
                "lm_head": (129280, 4096, 1)}


def bench_dense(args, dev):
    """MXFP8 projections (csrc/dense_mx.cu) vs cuBLAS BF16 at the model's decode shapes: one CUDA-graph
    replay per sample with L2 flushed before it (the weights stream from HBM, as in a decode step)."""
    from packmla.ops import check_errors
    from packmla.ops import dense as dense_ops

    T = args.tokens
    rows = []
    flush = L2Flush(dev)
    peak, tag = measured_hbm_gbs()
    for name, (N, K, B) in DENSE_SHAPES.items():
        g = torch.Generator(device=dev).manual_seed(N + K)
        w = torch.randn(B, N, K, device=dev, generator=g, dtype=torch.bfloat16) * K ** -0.5
        x = torch.randn(B, T, K, device=dev, generator=g, dtype=torch.bfloat16)
        wq = dense_ops.quantize_weight(w)
        y = torch.empty(B, T, N, dtype=torch.bfloat16, device=dev)
        y2 = torch.empty(B, T, N, dtype=torch.bfloat16, device=dev)
        mx = time_op(lambda: dense_ops.mx_linear(x, wq, out=y), args.rounds, args.warmup, dev, flush, graph=True)
        bf = time_op(lambda: torch.bmm(x, w.transpose(1, 2), out=y2), args.rounds, args.warmup, dev, flush, graph=True)
        check_errors(dev)
        rel = ((y.float() - y2.float()).norm() / y2.float().norm()).item()
        mx_bytes, bf_bytes = wq.codes.numel() + wq.scales.numel(), w.numel() * 2
        rows.append({"proj": name, "N": N, "K": K, "batch": B, "tokens": T,
                     "splits": dense_ops.choose_splits(T, N, K, B), "mxfp8_us": round(mx, 2),
                     "cublas_bf16_us": round(bf, 2), "speedup": round(bf / mx, 2),
                     "mxfp8_hbm_fraction": round(mx_bytes / mx / 1e3 / peak, 3),
                     "cublas_hbm_fraction": round(bf_bytes / bf / 1e3 / peak, 3), "rel_diff_vs_bf16": round(rel, 4)})
        del w, wq, x, y, y2
        torch.cuda.empty_cache()
    tot_mx = sum(r["mxfp8_us"] for r in rows)
    tot_bf = sum(r["cublas_bf16_us"] for r in rows)
    return {"case": "dense_projections", "tokens": T, "rows": rows, "sum_mxfp8_us": round(tot_mx, 1),
            "sum_cublas_bf16_us": round(tot_bf, 1), "peak_note": tag}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["moe", "decode", "store", "index", "dense", "decode-suite", "decode-paired",
                                     "fp4-suite", "glm-suite", "judge"],
                    help="decode-suite: native vs direct at batch 1/16/64, 128 heads, 32k and 128k contexts, "
                         "top-k 2048 (one JSON line per case)")
    ap.add_argument("--tokens", type=int, default=40)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--topk", type=int, default=None)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--heads", type=int, default=128)
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--swa", type=int, default=128, help="decode: SWA rows per query (0 = selected records only)")
    ap.add_argument("--kv-format", default="direct", choices=["direct", "native", "adapter", "fp4-native",
                                                              "fp4-direct"])
    ap.add_argument("--rows", type=int, default=24)
    ap.add_argument("--rounds", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--precision", default="default", choices=["default", "bf16"])
    ap.add_argument("--prof", action="store_true", help="report kernel phase / wait-time counters")
    ap.add_argument("--splits", type=int, default=0, help="decode: KV splits (0 = the automatic choice)")
    ap.add_argument("--paired", action="store_true", help="decode-suite: native and direct in paired rounds")
    ap.add_argument("--protocol", default="cold", choices=["cold", "reference"],
                    help="decode: 'cold' times one graph replay per sample with L2 flushed before it; 'reference' "
                         "times 100 back-to-back replays per sample without a flush, as the reference's decode "
                         "microbenchmark does")
    ap.add_argument("--with-adapter", action="store_true", help="decode-paired: add the adapter mode")
    ap.add_argument("--results", default=None, help="judge: the JSON lines of a decode-suite run")
    ap.add_argument("--out", default=None, help="glm-suite: append the rows to this JSON-lines file (with a "
                                                 "manifest of the sources, library and fixture)")
    ap.add_argument("--resume", action="store_true", help="glm-suite: continue --out, skipping recorded cases; "
                                                          "the manifest must match the current identity")
    ap.add_argument("--glm-batches", default=",".join(map(str, GLM_SUITE_BATCHES)),
                    help="glm-suite: comma-separated batches")
    args = ap.parse_args(argv)
    if args.case == "judge":
        with open(args.results) as f:
            rows = [json.loads(x) for x in f if x.strip().startswith("{")]
        verdict = judge(rows, args.rounds, paired=args.paired)
        print(json.dumps(verdict))
        if not verdict["passed"]:
            raise SystemExit("suite rejected")
        return verdict
    dev = torch.device("cuda", 0)
    if args.case == "moe":
        args.topk = args.topk or 8
        out = bench_moe(args, dev)
    elif args.case == "decode":
        args.topk = args.topk or 2048
        out = bench_decode(args, dev)
    elif args.case == "index":
        out = bench_index(args, dev)
    elif args.case == "dense":
        out = bench_dense(args, dev)
    elif args.case == "decode-paired":
        args.topk = args.topk or 2048
        modes = ("native", "direct", "adapter") if args.with_adapter else ("native", "direct")
        print(json.dumps(bench_decode_paired(args, dev, modes)), flush=True)
        return
    elif args.case == "fp4-suite":
        # the V4.1 FP4 decode table: H64, one query token, K512, SWA128, batches 8-32, FP4 Native and Packed
        args.topk, args.heads, args.swa = args.topk or 512, 64, 128
        for batch in FP4_SUITE_BATCHES:
            for fmt in ("fp4-native", "fp4-direct"):
                args.batch, args.kv_format = batch, fmt
                row = bench_decode(args, dev)
                row["clocks"] = dict(LAST_CLOCKS)
                print(json.dumps(row), flush=True)
                torch.cuda.empty_cache()
        return
    elif args.case == "glm-suite":
        args.heads = 16 if args.heads == 128 else args.heads
        args.context = 131076 if args.context == 32768 else args.context
        args.glm_batches = [int(x) for x in str(args.glm_batches).split(",") if x]
        bench_glm(args, dev)
        return
    elif args.case == "decode-suite":
        args.topk = args.topk or 2048
        args.heads = 128
        for ctx in (32768, 131072):
            for batch in (1, 16, 64):
                if args.paired:
                    args.context, args.batch = ctx, batch
                    print(json.dumps(bench_decode_paired(args, dev)), flush=True)
                    torch.cuda.empty_cache()
                    continue
                for fmt in ("native", "direct"):
                    args.context, args.batch, args.kv_format = ctx, batch, fmt
                    row = bench_decode(args, dev)
                    row["clocks"] = dict(LAST_CLOCKS)
                    print(json.dumps(row), flush=True)
                    torch.cuda.empty_cache()
        return
    else:
        out = bench_store(args, dev)
    out["clocks"] = dict(LAST_CLOCKS)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

"""CPU, multi-process (gloo): tensor/expert-parallel sharding reproduces the single-rank model.

Two ranks each hold a TP=EP=2 shard of the tiny model (heads, output-projection groups, routed experts
and the shared expert's intermediate are split; attention's latent KV is replicated) and exchange the
two per-layer partial sums through the communicator's all-reduce.  Rank 0's prefill and decode logits
must match the unsharded model.
"""
import os
import socket

import torch
import torch.multiprocessing as mp

from packmla.config import EngineConfig, ModelConfig
from packmla.kv.pool import KVPool
from packmla.models.v4flash import V4FlashModel
from packmla.models.weights import init_weights


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(cfg, rank: int, world: int, toks: torch.Tensor):
    from packmla.parallel.comm import TPComm

    W = init_weights(cfg, rank, world)
    pool = KVPool(cfg, EngineConfig(kv_cache_format="direct", device="cpu", tp=world, ep=world), 16, 2, 1024, "cpu")
    m = V4FlashModel(cfg, W, pool, TPComm() if world > 1 else None)
    slot = pool.admit(300)
    pre = m.prefill(toks[:250], 0, slot)
    dec = m.decode(toks[250:251], torch.tensor([250]), torch.tensor([slot]))[0]
    return pre, dec


def _worker(rank: int, world: int, port: int, out_path: str):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.tiny(num_layers=3)
        toks = torch.randint(0, cfg.vocab_size, (251,), generator=torch.Generator().manual_seed(7))
        pre, dec = _run(cfg, rank, world, toks)
        if rank == 0:
            torch.save({"pre": pre, "dec": dec}, out_path)
    finally:
        dist.destroy_process_group()


def test_tp2_matches_single_rank(tmp_path):
    cfg = ModelConfig.tiny(num_layers=3)
    toks = torch.randint(0, cfg.vocab_size, (251,), generator=torch.Generator().manual_seed(7))
    ref_pre, ref_dec = _run(cfg, 0, 1, toks)
    out = str(tmp_path / "tp2.pt")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    got = torch.load(out)
    rels = [((a.float() - b.float()).norm() / b.float().norm()).item()
            for a, b in ((got["pre"], ref_pre), (got["dec"], ref_dec))]
    print("tp2 vs single-rank relative error (prefill, decode):", rels)
    # each rank's partial sums are rounded to bf16 before the all-reduce (one rank adds its fp32 expert
    # sum directly), which the random model amplifies from layer to layer
    assert max(rels) < 4e-2, rels


def _serve_worker(rank: int, world: int, port: int, out_path: str, dp: bool = False):
    import torch.distributed as dist

    from packmla.config import EngineConfig
    from packmla.engine.engine import Engine, SamplingParams
    from packmla.parallel.comm import TPComm
    from packmla.server.driver import EngineDriver

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.tiny(num_layers=2)
        ecfg = EngineConfig(device="cpu", tp=world, ep=world, chunked_prefill_size=64, max_running_requests=4,
                            cuda_graph_bs=[1, 2, 4], dp_attention=dp)
        eng = Engine.build(cfg, ecfg, "cpu", rank, world, TPComm(), max_context=512)
        drv = EngineDriver(eng, rank, world, cpu_group=dist.new_group(backend="gloo"))
        if rank == 0:
            drv.start()
            streams = [drv.submit(p, SamplingParams(max_new_tokens=4)) for p in ([1, 5, 9, 12], [1, 7] * 40)]
            for st in streams:
                assert st.done.wait(120)
            toks = [st.tokens for st in streams]
            drv.stop()
            torch.save({"tokens": toks, "metrics": eng.metrics.snapshot()}, out_path)
        else:
            drv.run_worker()
            torch.save({"metrics": eng.metrics.snapshot()}, out_path + ".r1")
    finally:
        dist.destroy_process_group()


def test_server_driver_keeps_tp_ranks_in_lockstep(tmp_path):
    out = str(tmp_path / "serve.pt")
    mp.spawn(_serve_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r0 = torch.load(out)
    r1 = torch.load(out + ".r1")
    assert [len(t) for t in r0["tokens"]] == [4, 4]
    for key in ("decode_steps", "prefill_tokens", "requests_finished"):
        assert r0["metrics"][key] == r1["metrics"][key], key


def test_server_driver_dp_attention_streams_every_ranks_tokens(tmp_path):
    """With DP attention the second request is served by rank 1; its tokens still reach rank 0's HTTP
    stream (gathered after every step), and each rank finished only the requests it owns."""
    out = str(tmp_path / "serve_dp.pt")
    mp.spawn(_serve_worker, args=(2, _free_port(), out, True), nprocs=2, join=True)
    r0 = torch.load(out)
    r1 = torch.load(out + ".r1")
    assert [len(t) for t in r0["tokens"]] == [4, 4]
    assert r0["metrics"]["requests_finished"] == 1 and r1["metrics"]["requests_finished"] == 1


def _ep_worker(rank: int, world: int, port: int, out_path: str):
    import torch.distributed as dist

    from packmla.parallel.ep import EPMoE, local_expert_fn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.tiny(num_layers=2)
        W = init_weights(cfg, rank, world)
        lw = W["layers"][1]
        h, ids, w = _ep_inputs(cfg, rank)
        res = {}
        for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            ep = EPMoE(cfg.n_routed_experts, combine_dtype=dt)
            res[name] = ep.forward(h, ids, w, local_expert_fn(lw, ep.expert_base, ep.local_experts,
                                                               cfg.expert_format))
        torch.save({**res, "counts": ep.last_counts}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def _ep_inputs(cfg, rank: int):
    g = torch.Generator().manual_seed(100 + rank)
    T = 37 + 11 * rank  # ranks hold different token counts
    h = torch.randn(T, cfg.hidden_size, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(cfg.n_routed_experts, generator=g)[:cfg.moe_topk] for _ in range(T)]).int()
    w = torch.rand(T, cfg.moe_topk, generator=g)
    return h, ids, w


def test_expert_parallel_dispatch_combine_matches_all_experts(tmp_path):
    """Token-sharded EP (all-to-all dispatch, local experts, all-to-all combine) over 2 gloo ranks equals
    one rank applying all experts to the same tokens."""
    from packmla.ops import moe as moe_ops

    out = str(tmp_path / "ep")
    mp.spawn(_ep_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    cfg = ModelConfig.tiny(num_layers=2)
    lw = init_weights(cfg)["layers"][1]
    for rank in range(2):
        got = torch.load(f"{out}.{rank}")
        h, ids, w = _ep_inputs(cfg, rank)
        ref = moe_ops.experts_reference(h, ids, w, lw["w13"], lw["w2"], 0, cfg.n_routed_experts)
        torch.testing.assert_close(got["fp32"], ref, atol=1e-4, rtol=1e-4)
        assert ((got["bf16"] - ref).norm() / ref.norm()).item() < 1e-2  # bf16 combine rows
        assert sum(got["counts"]["sent"]) == h.shape[0] * cfg.moe_topk


def _capture_worker(rank: int, world: int, port: int, out_dir: str):
    import torch.distributed as dist

    from packmla.parallel.comm import TPComm
    from packmla.training.data.capture import capture_cache

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        capture_cache(os.path.join(out_dir, "tp2"), ModelConfig.tiny(num_layers=2), issues=3, development=1,
                      train_queries=1, dev_queries=1, prompt_len=64, comm=TPComm())
    finally:
        dist.destroy_process_group()


def test_tp2_capture_gathers_all_heads(tmp_path):
    """Capture under TP=2: every query state holds all heads (gathered in rank order) and matches the
    single-rank capture of the same model; only rank 0 writes the cache."""
    from packmla.training.data.cache import load_cached_layer
    from packmla.training.data.capture import capture_cache

    cfg = ModelConfig.tiny(num_layers=2)
    capture_cache(tmp_path / "tp1", cfg, issues=3, development=1, train_queries=1, dev_queries=1, prompt_len=64)
    mp.spawn(_capture_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    layer = cfg.c4_layers[0]
    one, two = load_cached_layer(tmp_path / "tp1", layer), load_cached_layer(tmp_path / "tp2", layer)
    for role in ("train", "development"):
        assert len(one[role]) == len(two[role]) > 0
        for a, b in zip(one[role], two[role]):
            assert b["q"].shape == (cfg.num_heads, 512) and b["sink"].shape == (cfg.num_heads,)
            assert torch.equal(a["sink"], b["sink"])  # replicated init, gathered in head order
            for k in ("q", "raw", "target"):
                rel = ((a[k] - b[k]).norm() / a[k].norm()).item()
                assert rel < 5e-2, (role, k, rel)


def _dp_run(cfg, rank: int, world: int, prompts: list[torch.Tensor]):
    """Rank r owns prompt r: prefills it while the other ranks run token-less forwards, then every
    rank decodes its own request in one step.  Returns this rank's (prefill logits, decode logits)."""
    from packmla.parallel.comm import TPComm

    W = init_weights(cfg, rank, world, dp_attention=True)
    pool = KVPool(cfg, EngineConfig(kv_cache_format="direct", device="cpu", tp=world, ep=world), 16, 2, 1024, "cpu")
    m = V4FlashModel(cfg, W, pool, TPComm())
    slot = pool.admit(300)
    pre = None
    for owner, toks in enumerate(prompts):
        counts = [0] * world
        counts[owner] = toks.shape[0] - 1
        m.dp_counts = counts
        if owner == rank:
            pre = m.prefill(toks[:-1], 0, slot)
        else:
            m.dp_idle_forward()
    m.dp_counts = [1] * world
    mine = prompts[rank]
    n = mine.shape[0] - 1
    dec = m.decode(mine[n:], torch.tensor([n]), torch.tensor([slot]))[0]
    return pre, dec


def _dp_worker(rank: int, world: int, port: int, out_path: str):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.tiny(num_layers=3)
        g = torch.Generator().manual_seed(11)
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (201, 137)]
        pre, dec = _dp_run(cfg, rank, world, prompts)
        torch.save({"pre": pre, "dec": dec}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_dp_attention_matches_single_rank(tmp_path):
    """DP attention over 2 ranks (each rank: its own request, every head, half the routed experts; tokens
    exchanged by all-gather / reduce-scatter in every MoE block, a token-less forward on the rank without
    a prefill) reproduces the single-rank model's logits for both requests."""
    cfg = ModelConfig.tiny(num_layers=3)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (201, 137)]
    W = init_weights(cfg)
    refs = []
    for toks in prompts:
        pool = KVPool(cfg, EngineConfig(kv_cache_format="direct", device="cpu"), 16, 2, 1024, "cpu")
        m = V4FlashModel(cfg, W, pool)
        slot = pool.admit(300)
        n = toks.shape[0] - 1
        pre = m.prefill(toks[:-1], 0, slot)
        dec = m.decode(toks[n:], torch.tensor([n]), torch.tensor([slot]))[0]
        refs.append((pre, dec))
    out = str(tmp_path / "dp2")
    mp.spawn(_dp_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for r in range(2):
        got = torch.load(f"{out}.{r}")
        rels = [((a.float() - b.float()).norm() / b.float().norm()).item()
                for a, b in ((got["pre"], refs[r][0]), (got["dec"], refs[r][1]))]
        print(f"dp2 rank {r} vs single rank (prefill, decode):", rels)
        assert max(rels) < 4e-2, rels


def _dp_engine_worker(rank: int, world: int, port: int, out_path: str):
    import torch.distributed as dist

    from packmla.engine.engine import Engine, SamplingParams
    from packmla.parallel.comm import TPComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig.tiny(num_layers=3)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 130, 5, 40, 90)]
        ecfg = EngineConfig(device="cpu", dp_attention=True, tp=world, ep=world, chunked_prefill_size=64,
                            max_running_requests=3, cuda_graph_bs=[1, 2, 3])
        eng = Engine.build(cfg, ecfg, "cpu", rank, world, TPComm(), max_context=512)
        rids = [eng.add_request(p, SamplingParams(max_new_tokens=6)) for p in prompts]
        steps = 0
        while eng.has_work():
            eng.step()
            steps += 1
        mine = {r: eng.result(r).output_ids for r in rids if eng.owns(r)}
        torch.save({"outputs": mine, "steps": steps, "free": eng.pool.pages.free == eng.pool.num_pages},
                   f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_dp_attention_engine_matches_single_rank(tmp_path):
    """The engine with DP attention over 2 ranks (requests spread by id, prefill steps where one rank has no
    chunk, decode batches padded to the larger rank's) produces the single-rank engine's greedy tokens."""
    from packmla.engine.engine import Engine, SamplingParams

    cfg = ModelConfig.tiny(num_layers=3)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 130, 5, 40, 90)]
    ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=6, cuda_graph_bs=[1, 2, 4, 6])
    ref = Engine.build(cfg, ecfg, "cpu", max_context=512).generate(prompts, SamplingParams(max_new_tokens=6))
    out = str(tmp_path / "dpe")
    mp.spawn(_dp_engine_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    got = [torch.load(f"{out}.{r}") for r in range(2)]
    assert got[0]["steps"] == got[1]["steps"]  # lockstep
    assert all(x["free"] for x in got)  # every page returned
    merged = {**got[0]["outputs"], **got[1]["outputs"]}
    assert sorted(merged) == list(range(len(prompts)))
    assert [merged[i] for i in range(len(prompts))] == ref

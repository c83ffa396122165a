"""Fused GEMM + all-reduce and one-kernel all-reduce (csrc/comm_fused.cu) against fp32 PyTorch.

One GPU: the kernels run with world = 1 (every tile owned by this rank), which exercises the GEMM,
the reduce-scatter/all-gather addressing and the flags; a fake second rank whose buffer nobody
serves makes every peer wait run out, which must be reported in the error word, not hang.
Two GPUs (skipped with fewer): NCCL-initialised ranks compare against the sum of all ranks' inputs
and against each other bitwise, and the tiny model under TP=2 against the single-rank model.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from packmla.ops._ext import check_errors, error_word, ext

pytestmark = pytest.mark.gpu


def _comm(hidden=4096, timeout_s=2.0):
    from packmla.parallel.fused import FusedComm

    return FusedComm(torch.device("cuda", 0), hidden, timeout_s=timeout_s)


@pytest.mark.parametrize("B,N,K", [(1, 4096, 1024), (7, 256, 128), (40, 4096, 4096), (300, 4096, 1024),
                                   (512, 1024, 512), (129, 2048, 2048), (80, 4096, 4096)])
def test_gemm_allreduce_world1(B, N, K):
    comm = _comm()
    g = torch.Generator(device="cuda").manual_seed(B * 7 + K)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    ref = x.float() @ w.float().T
    try:
        for s in (1, 2, 4, 8):
            if K % (64 * s) or (N // 256) * -(-B // 128) * s > comm.num_sms:
                continue
            for one_shot in (True, False):
                out = comm.gemm_all_reduce(x, w, splits=s, one_shot=one_shot)
                check_errors(torch.device("cuda", 0))
                rel = ((out.float() - ref).norm() / ref.norm()).item()
                assert rel < 8e-3, (s, one_shot, rel)
    finally:
        comm.close()


@pytest.mark.parametrize("n", [4096, 8 * 4096, 40 * 4096 + 8, 512 * 4096])
def test_allreduce_world1_exact(n):
    comm = _comm()
    g = torch.Generator(device="cuda").manual_seed(n)
    a = torch.randn(n, device="cuda", generator=g).bfloat16()
    f = torch.randn(n, device="cuda", generator=g)
    try:
        for one_shot in (True, False):
            out = comm.all_reduce_sum(f, a, one_shot=one_shot)
            check_errors(torch.device("cuda", 0))
            assert torch.equal(out, (a.float() + f).bfloat16())
        out2 = comm.all_reduce(a.clone())
        check_errors(torch.device("cuda", 0))
        assert torch.equal(out2, a)
    finally:
        comm.close()


def test_fused_calls_replay_in_cuda_graph():
    comm = _comm()
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(24, 1024, device="cuda", generator=g).bfloat16()
    w = (torch.randn(4096, 1024, device="cuda", generator=g) / 32).bfloat16()
    f = torch.randn(24, 4096, device="cuda", generator=g)
    try:
        comm.gemm_all_reduce(x, w)  # warm-up outside capture
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                y = comm.gemm_all_reduce(x, w)
                z = comm.all_reduce_sum(f, y)
        torch.cuda.current_stream().wait_stream(s)
        e0 = int(comm.epoch[0].item())
        for i in range(5):
            x.copy_(torch.randn(24, 1024, device="cuda", generator=g).bfloat16())
            graph.replay()
            torch.cuda.synchronize()
            check_errors(torch.device("cuda", 0))
            ref = (x.float() @ w.float().T).bfloat16()
            assert ((y.float() - ref.float()).norm() / ref.float().norm()).item() < 8e-3
            assert torch.equal(z, (y.float() + f).bfloat16())
        assert int(comm.epoch[0].item()) == e0 + 10  # two launches per replay
        del graph
    finally:
        comm.close()


def test_peer_wait_times_out_with_error_status():
    """A second 'rank' that never runs: every wait on it must give up and report kPeerTimeout (4)."""
    from packmla.parallel.fused import FusedComm, SymmetricBuffer

    comm = FusedComm(torch.device("cuda", 0), 1024, timeout_s=0.05)
    ghost = SymmetricBuffer(comm.buf.nbytes, torch.device("cuda", 0))
    err = error_word(torch.device("cuda", 0))
    try:
        peers = torch.tensor([comm.buf.ptr, ghost.ptr], dtype=torch.int64, device="cuda")
        layout = list(comm.layout)
        layout[5] = max(layout[5], 2)
        a = torch.ones(8192, dtype=torch.bfloat16, device="cuda")
        out = torch.empty_like(a)
        ext().allreduce(a, None, out, peers, 0, 2, layout, comm.epoch, err, 2048, 1, int(0.05e9))
        torch.cuda.synchronize()
        vals = err.tolist()
        assert vals[0] == 4 and vals[3] >= 1, vals
        err.zero_()
        # the context is still usable
        y = comm.all_reduce(a.clone())
        check_errors(torch.device("cuda", 0))
        assert torch.equal(y, a)
    finally:
        err.zero_()
        ghost.close()
        comm.close()


# ----------------------------------------------------------------------------- 2, 4 and 8 GPUs
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mp_worker(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from packmla.parallel.fused import FusedComm

    comm = FusedComm(dev, 4096, timeout_s=5.0)
    res = {}
    try:
        for B, K in ((1, 1024), (40, 4096), (300, 1024)):
            xs = [torch.randn(B, K, generator=torch.Generator().manual_seed(100 * r + B)).bfloat16() for r in range(world)]
            ws = [(torch.randn(4096, K, generator=torch.Generator().manual_seed(1000 * r + K)) / K ** 0.5).bfloat16()
                  for r in range(world)]
            ref = sum(x.float() @ w.float().T for x, w in zip(xs, ws))
            fs = [torch.randn(B, 4096, generator=torch.Generator().manual_seed(7 * r + B)) for r in range(world)]
            for one_shot in (True, False):
                y = comm.gemm_all_reduce(xs[rank].to(dev), ws[rank].to(dev), one_shot=one_shot)
                torch.cuda.synchronize()
                res[f"gemm_{B}_{K}_{one_shot}"] = (y.cpu(), ref)
                z = comm.all_reduce_sum(fs[rank].to(dev), y, one_shot=one_shot)
                torch.cuda.synchronize()
                res[f"ar_{B}_{one_shot}"] = (z.cpu(), sum(f for f in fs) + world * y.cpu().float())
        check_errors(dev)
        torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        comm.close()
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_collectives_multi_gpu(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_mp_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    for key, (y0, ref) in res[0].items():
        for r in range(1, world):
            assert torch.equal(y0, res[r][key][0]), (key, r)  # every rank receives the same bits
        rel = ((y0.float() - ref).norm() / ref.norm()).item()
        assert rel < 1e-2, (key, rel)


def _run_model(eng, dev):
    cfg = eng.cfg
    toks = torch.randint(0, cfg.vocab_size, (251,), generator=torch.Generator().manual_seed(7)).to(dev)
    slot = eng.pool.admit(300)
    pre = eng.model.prefill(toks[:250], 0, slot)
    dec = eng.model.decode(toks[250:251], torch.tensor([250], device=dev), torch.tensor([slot], device=dev))[0]
    eng.pool.release(slot)
    return pre.float().cpu(), dec.float().cpu()


def _engine(rank, world, comm, dev):
    from helpers import small_gpu_config

    from packmla.config import EngineConfig
    from packmla.engine.engine import Engine

    cfg = small_gpu_config(o_groups=8)  # output groups split over up to 8 ranks
    ecfg = EngineConfig(kv_cache_format="direct", tp=world, ep=world, max_running_requests=2, cuda_graph_bs=[1],
                        disable_cuda_graph=True, moe_precision="bf16")
    return Engine.build(cfg, ecfg, dev, rank, world, comm, max_context=1024, max_requests=2, kv_bytes=64 << 20)


def _model_worker(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch.distributed as dist

    from packmla.parallel.comm import TPComm
    from packmla.parallel.fused import FusedComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from helpers import small_gpu_config

    comm = FusedComm(dev, small_gpu_config(o_groups=8).hidden_size, timeout_s=5.0)
    try:
        eng = _engine(rank, world, comm, dev)
        fused = _run_model(eng, dev)
        eng.model.comm = TPComm()  # same shards, NCCL all-reduces
        eng.model.ar_hook = None
        nccl = _run_model(eng, dev)
        check_errors(dev)
        if rank == 0:
            torch.save({"fused": fused, "nccl": nccl, "fallbacks": comm.fallbacks}, os.path.join(out_dir, "m.pt"))
    finally:
        comm.close()
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_model_tp_fused_matches_single_rank(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    dev = torch.device("cuda", 0)
    eng = _engine(0, 1, None, dev)
    ref = _run_model(eng, dev)
    del eng
    torch.cuda.empty_cache()
    mp.spawn(_model_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = torch.load(tmp_path / "m.pt")
    assert got["fallbacks"] == 0
    rel = {}
    for name in ("fused", "nccl"):
        rel[name] = [((a - b).norm() / b.norm()).item() for a, b in zip(got[name], ref)]
    print(f"TP{world} vs single-rank relative error (prefill, decode):", rel)
    # partial sums are rounded to bf16 before either all-reduce; the random model amplifies it per layer
    assert max(rel["fused"]) < 6e-2 and max(rel["nccl"]) < 6e-2, rel

"""CPU: failure detection on the host (no GPU fault is ever provoked).

* a step that raises marks the engine failed: open streams end with "error", /health turns 503,
  new requests are refused;
* a step that outlives the watchdog turns /health 503 while it runs;
* a TP rank that dies between steps: the surviving rank's next CPU-group collective fails and its
  driver reports the failure instead of hanging (gloo ranks, short process-group timeout).
"""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp
from fastapi.testclient import TestClient

from packmla.config import EngineConfig, ModelConfig
from packmla.engine.engine import Engine, SamplingParams
from packmla.server.app import create_app
from packmla.server.driver import EngineDriver
from packmla.server.tokenizer import ByteTokenizer


def _engine(rank=0, world=1, comm=None):
    cfg = ModelConfig.tiny(num_layers=2)
    ecfg = EngineConfig(device="cpu", tp=world, ep=world, chunked_prefill_size=64, max_running_requests=2,
                        cuda_graph_bs=[1, 2])
    return Engine.build(cfg, ecfg, "cpu", rank, world, comm, max_context=512)


def test_step_exception_fails_requests_and_health():
    def hook(step):
        if step == 3:
            raise RuntimeError("injected step failure")

    eng = _engine()
    drv = EngineDriver(eng, fault_hook=hook).start()
    client = TestClient(create_app(drv, ByteTokenizer(eng.cfg.vocab_size), "tiny"))
    r = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 8, "ignore_eos": True})
    assert r.status_code == 500 and "injected" in r.text
    assert client.get("/health").status_code == 503
    assert client.post("/v1/completions", json={"prompt": "x", "max_tokens": 1}).status_code == 503
    assert eng.metrics.snapshot()["engine_failures"] == 1
    drv.stop()


def test_watchdog_marks_slow_step_unhealthy():
    def hook(step):
        if step == 1:
            time.sleep(1.5)

    eng = _engine()
    drv = EngineDriver(eng, watchdog_s=0.3, fault_hook=hook).start()
    client = TestClient(create_app(drv, ByteTokenizer(eng.cfg.vocab_size), "tiny"))
    st = drv.submit([1, 5, 6], SamplingParams(max_new_tokens=4, ignore_eos=True))
    seen = set()
    t0 = time.time()
    while not st.done.is_set() and time.time() - t0 < 30:
        seen.add(client.get("/health").status_code)
        time.sleep(0.05)
    assert st.finish_reason == "length" and 503 in seen
    assert client.get("/health").status_code == 200
    drv.stop()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from packmla.parallel.comm import TPComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    eng = _engine(rank, world, TPComm())
    group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=20))

    def die(step):  # rank 1 leaves between steps, with nothing in flight
        if rank == 1 and step == 2:
            os._exit(17)

    drv = EngineDriver(eng, rank, world, group, fault_hook=die)
    if rank == 0:
        drv.start()
        st = drv.submit([1, 9, 9, 9], SamplingParams(max_new_tokens=16, ignore_eos=True))
        t0 = time.time()
        done = st.done.wait(120)
        torch.save({"done": done, "reason": st.finish_reason, "error": repr(drv.error),
                    "seconds": time.time() - t0}, os.path.join(out_dir, "r0.pt"))
        os._exit(0)
    drv.run_worker()


def test_dead_rank_is_detected_by_the_survivor(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes[1] == 17, codes
    res = torch.load(tmp_path / "r0.pt")
    assert res["done"] and res["reason"] == "error" and res["error"] != "None", res
    assert res["seconds"] < 60

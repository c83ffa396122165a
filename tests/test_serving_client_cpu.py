"""CPU: the serving benchmark client against a live packmla HTTP server (tiny model, HiCache on)."""
import socket
import threading
import time

import pytest

from packmla.config import EngineConfig, ModelConfig
from packmla.engine.engine import Engine
from packmla.server.app import create_app
from packmla.server.driver import EngineDriver
from packmla.server.tokenizer import ByteTokenizer


@pytest.fixture(scope="module")
def server_url():
    import uvicorn

    cfg = ModelConfig.tiny(num_layers=2)
    ecfg = EngineConfig(device="cpu", chunked_prefill_size=128, max_running_requests=4, cuda_graph_bs=[1, 2, 4],
                        enable_hierarchical_cache=True)
    eng = Engine.build(cfg, ecfg, "cpu", max_context=1024)
    driver = EngineDriver(eng).start()
    app = create_app(driver, ByteTokenizer(cfg.vocab_size), "tiny")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.05)
    yield f"http://127.0.0.1:{port}", eng
    server.should_exit = True
    th.join(10)
    driver.stop()


def test_random_dataset_protocol(server_url):
    from packmla.bench.serving import bench

    url, eng = server_url
    out = bench(url, "random", input_len=100, output_len=6, concurrency=2, flush_cache=True)
    for phase, n in (("warmup", 2), ("measured", 6)):
        assert out[phase]["completed"] == n and out[phase]["success_rate"] == 1.0, out[phase]
        assert out[phase]["total_output_tokens"] == 6 * n
        assert out[phase]["ttft_ms"]["mean"] > 0
    assert out["server"]["kv_cache_format"] == "direct"


def test_multi_turn_hits_host_cache(server_url):
    from packmla.bench.serving import bench

    url, eng = server_url
    before = eng.metrics.snapshot().get("hicache_hit_tokens", 0)
    out = bench(url, "multi-turn", input_len=80, output_len=4, concurrency=2, turns=3, sessions=2)
    assert [t["success_rate"] for t in out["turns"]] == [1.0, 1.0, 1.0]
    assert eng.metrics.snapshot().get("hicache_hit_tokens", 0) > before

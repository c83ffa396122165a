"""CPU: the server launcher accepts the reference launcher's flags and maps them onto packmla's options."""
import json

import pytest

from packmla.config import EngineConfig
from packmla.server.__main__ import build_parser, resolve_args

GRAPHS = {"decode": {"backend": "full", "max_bs": 136, "bs": [1, 2, 4, 8, 16]}, "prefill": {"backend": "disabled"}}


def _resolve(*argv):
    args = build_parser().parse_args(list(argv))
    return args, resolve_args(args)


def test_reference_launch_line_maps_onto_engine_config():
    args, kw = _resolve("--model-path", "v4-flash", "--tp", "4", "--ep", "4", "--kv-cache-dtype", "fp8_e4m3",
                        "--cuda-graph-config", json.dumps(GRAPHS), "--watchdog-timeout", "1800",
                        "--moe-runner-backend", "flashinfer_mxfp4", "--dsv4-c4-cache-format", "remnant",
                        "--dsv4-c4-cache-implementation", "kernel", "--dsv4-c4-cache-keep-count", "256",
                        "--enable-hierarchical-cache", "--hicache-ratio", "2.0", "--hicache-write-policy",
                        "write_through", "--hicache-io-backend", "kernel", "--hicache-mem-layout", "layer_first",
                        "--enable-metrics", "--log-requests", "--random-seed", "7", "--max-running-requests", "40",
                        "--device", "cpu")
    assert args.model == "v4-flash" and args.seed == 7 and args.watchdog_timeout == 1800
    assert kw["kv_cache_format"] == "direct" and kw["decode_impl"] == "direct" and kw["keep_count"] == 256
    assert kw["cuda_graph_bs"] == [1, 2, 4, 8, 16] and kw["disable_cuda_graph"]  # CPU: no graphs
    assert kw["prefix_cache"] and not _resolve("--disable-radix-cache")[1]["prefix_cache"]
    assert kw["hicache_mem_layout"] == "layer_first"
    EngineConfig(tp=4, ep=4, enable_hierarchical_cache=True, **kw).validate()


def test_selectors_and_rejections():
    _, kw = _resolve("--dsv4-c4-cache-format", "native", "--device", "cuda",
                     "--cuda-graph-config", json.dumps({"decode": {"backend": "disabled"}}))
    assert kw["kv_cache_format"] == "native" and kw["disable_cuda_graph"]
    _, kw = _resolve("--dsv4-c4-cache-implementation", "adapter", "--device", "cuda")
    assert kw["decode_impl"] == "adapter" and not kw["disable_cuda_graph"]
    with pytest.raises(SystemExit):
        _resolve("--tp", "2", "--ep", "4")
    _, kw = _resolve("--dsv4-c4-cache-layer-keep-counts", "2:256,4:192")
    assert kw["layer_keep_counts"] == {2: 256, 4: 192}
    with pytest.raises(ValueError):  # a non-256 layout is read by reconstruction only
        EngineConfig(**kw).validate()
    _, kw = _resolve("--dsv4-c4-cache-layer-keep-counts", "2:256,4:192", "--dsv4-c4-cache-implementation", "adapter")
    EngineConfig(**kw).validate()
    with pytest.raises(SystemExit):  # unsupported choice
        _resolve("--moe-runner-backend", "deep_gemm")
    _, kw = _resolve("--dsv4-c4-cache-keep-count", "192")
    with pytest.raises(ValueError):  # Direct serving keeps 256 survivors only
        EngineConfig(**kw).validate()


def test_request_log_and_metric_export(tmp_path, caplog):
    import logging

    from packmla.config import ModelConfig
    from packmla.engine.engine import Engine, SamplingParams
    from packmla.server.__main__ import request_logger
    from packmla.server.driver import EngineDriver

    args, _ = _resolve("--log-requests", "--log-requests-level", "3", "--export-metrics-to-file",
                       "--export-metrics-to-file-dir", str(tmp_path / "m"), "--device", "cpu")
    rl = request_logger(args)
    assert rl.log_requests and rl.log_level == 3 and rl.export_dir == str(tmp_path / "m")
    assert request_logger(_resolve("--device", "cpu")[0]) is None
    with pytest.raises(SystemExit):  # export without a directory
        request_logger(_resolve("--export-metrics-to-file")[0])
    cfg = ModelConfig.tiny(num_layers=2)
    eng = Engine.build(cfg, EngineConfig(device="cpu", max_running_requests=2, cuda_graph_bs=[1, 2]), "cpu",
                       max_context=256)
    driver = EngineDriver(eng, request_logger=rl).start()
    try:
        with caplog.at_level(logging.INFO, logger="packmla.requests"):
            for n in (3, 5):
                driver.generate([5, 6, 7, 8], SamplingParams(max_new_tokens=n))
    finally:
        driver.stop()
    files = list((tmp_path / "m").glob("request-metrics-*.jsonl"))
    assert len(files) == 1
    recs = [json.loads(line) for line in files[0].read_text().splitlines()]
    assert [r["completion_tokens"] for r in recs] == [3, 5] and all(r["finish_reason"] == "length" for r in recs)
    assert recs[1]["prompt_ids"] == [5, 6, 7, 8] and len(recs[1]["output_ids"]) == 5
    assert recs[1]["sampling_params"]["max_new_tokens"] == 5
    assert all(r["ttft_s"] is not None and r["e2e_s"] >= r["ttft_s"] for r in recs) and recs[1]["tpot_s"] > 0
    assert sum("request finished" in m for m in caplog.messages) == 2

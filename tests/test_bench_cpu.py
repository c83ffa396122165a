"""CPU: host-side logic of the benchmark harnesses (paired-round ordering and ratios)."""
import math

import pytest

from packmla.bench.microbench import paired_rounds


def test_paired_rounds_rotate_order_and_report_ratios():
    calls = []
    times = {"native": iter([10.0, 10.0, 12.0]), "direct": iter([11.0, 9.0, 12.0]), "adapter": iter([20.0] * 3)}

    def timer(m):
        def run():
            calls.append(m)
            return next(times[m])
        return run

    out = paired_rounds({m: timer(m) for m in ("native", "direct", "adapter")}, 3)
    assert calls == ["native", "direct", "adapter", "direct", "adapter", "native", "adapter", "native", "direct"]
    assert out["mean_us"] == {"native": round(32 / 3, 3), "direct": round(32 / 3, 3), "adapter": 20.0}
    r = out["ratio"]["direct/native"]
    assert r["geomean"] == round(math.exp((math.log(1.1) + math.log(0.9) + 0.0) / 3), 5)
    assert r["min"] == 0.9 and r["max"] == 1.1 and out["baseline"] == "native"
    with pytest.raises(ValueError):
        paired_rounds({}, 3)


def _suite(rounds=30, clocks=None):
    from packmla.bench.microbench import SUITE_BATCHES, SUITE_CONTEXTS, SUITE_FORMATS

    clk = clocks or {"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": []}
    return [{"case": "sparse_mla_decode", "context": c, "batch": b, "kv_format": f, "us": 50.0, "rounds": rounds,
             "clocks": dict(clk)} for c in SUITE_CONTEXTS for b in SUITE_BATCHES for f in SUITE_FORMATS]


def test_judge_accepts_a_complete_clean_suite(tmp_path):
    import json

    from packmla.bench import microbench

    path = tmp_path / "suite.jsonl"
    path.write_text("".join(json.dumps(r) + "\n" for r in _suite()))
    v = microbench.main(["judge", "--results", str(path)])
    assert v["passed"] and v["cases"] == v["expected"] == 12


def test_judge_rejects_missing_short_slow_and_locked_runs():
    from packmla.bench.microbench import judge

    rows = _suite()
    v = judge(rows[:-1], 30)
    assert not v["passed"] and v["missing"] == [[131072, 64, "direct"]]
    assert not judge(_suite(rounds=10), 30)["passed"]
    v = judge(_suite(clocks={"sm_mhz": 1500.0, "sm_max_mhz": 1965.0, "reasons": ["hw_thermal_slowdown"]}), 30)
    assert not v["passed"] and "hw_thermal_slowdown" in v["rejected"][0]["reason"]
    v = judge(_suite(clocks={"sm_mhz": 1000.0, "sm_max_mhz": 1965.0, "reasons": []}), 30)
    assert not v["passed"] and "well below" in v["rejected"][0]["reason"]
    v = judge(_suite(clocks={"sm_mhz": 1300.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}), 30)
    assert v["passed"] and len(v["notes"]) == 12  # power capping is kept and noted
    bad = _suite()
    bad[3]["us"] = float("nan")
    assert not judge(bad, 30)["passed"]
    assert not judge(_suite() + _suite()[:1], 30)["passed"]  # a duplicate case


def test_validation_tier_of_a_diff():
    from packmla.utils.validation_tier import classify, main

    assert classify(["README.md", "tests/test_codec.py"])["tier"] == "low"
    assert classify(["packmla/server/app.py", "packmla/engine/engine.py"])["tier"] == "medium"
    out = classify(["packmla/training/train.py", "csrc/kv_store.cu"])
    assert out["tier"] == "high" and out["files"]["packmla/training/train.py"] == "low"
    assert any("ncu" in c for c in out["required"])
    assert classify([])["tier"] == "low"
    assert main(["bench.py"])["tier"] == "medium"


def _hold_lock(root, ready, release):
    from packmla.utils.build_lock import build_lock

    with build_lock(root):
        ready.set()
        release.wait(30)


def test_build_lock_is_exclusive_and_released_on_exit(tmp_path):
    import multiprocessing as mp

    from packmla.utils.build_lock import BuildLocked, build_lock

    ctx = mp.get_context("spawn")
    ready, release = ctx.Event(), ctx.Event()
    p = ctx.Process(target=_hold_lock, args=(str(tmp_path), ready, release))
    p.start()
    try:
        assert ready.wait(60)
        with pytest.raises(BuildLocked, match="pid"):
            with build_lock(str(tmp_path), timeout_s=0.5, poll_s=0.1):
                pass
    finally:
        release.set()
        p.join(30)
    with build_lock(str(tmp_path), timeout_s=5):  # free again once the holder is gone
        pass


def test_source_digest_record_detects_a_stale_library(tmp_path):
    from packmla.utils.source_digest import check_record, source_digest, write_record

    (tmp_path / "csrc" / "common").mkdir(parents=True)
    (tmp_path / "packmla").mkdir()
    (tmp_path / "csrc" / "k.cu").write_text("kernel v1")
    (tmp_path / "csrc" / "common" / "h.cuh").write_text("header")
    (tmp_path / "setup.py").write_text("setup")
    assert check_record(str(tmp_path)) is None  # no record yet: nothing to compare
    d = write_record(str(tmp_path))
    assert check_record(str(tmp_path)) is None and d == source_digest(str(tmp_path))
    (tmp_path / "csrc" / "common" / "h.cuh").write_text("header v2")
    assert "rebuild" in check_record(str(tmp_path))


def _sweep_dir(root, name, points):
    import json

    d = root / name
    d.mkdir()
    pts = [{"concurrency": c, "repeat": r, "successful_requests_per_s": rps, "output_throughput_tok_s": tok,
            "ttft_ms": {"p90": p90}, "passed": True, "success_rate": 1.0} for c, r, rps, tok, p90 in points]
    (d / "summary.json").write_text(json.dumps({"points": pts, "stopped": None}))
    return d


def test_analyze_pairs_points_and_reports_geomean(tmp_path):
    import math

    from packmla.bench import analyze

    a = _sweep_dir(tmp_path, "native", [(20, 1, 1.0, 100.0, 500.0), (24, 1, 2.0, 200.0, 800.0), (28, 1, 2.5, 250, 900)])
    b = _sweep_dir(tmp_path, "direct", [(20, 1, 1.1, 110.0, 450.0), (24, 1, 2.4, 220.0, 800.0), (32, 1, 3.0, 300, 1e3)])
    out = analyze.main([str(a), str(b), "--output", str(tmp_path / "cmp.json")])
    assert [p["concurrency"] for p in out["points"]] == [20, 24]
    assert math.isclose(out["geomean_ratio"]["successful_requests_per_s"], math.sqrt(1.1 * 1.2))
    assert math.isclose(out["geomean_ratio"]["ttft_p90_ms"], math.sqrt(0.9 * 1.0))
    assert out["only_baseline"] == [[28, 1]] and out["only_candidate"] == [[32, 1]]
    assert (tmp_path / "cmp.json").exists()


def test_latency_histograms_export_cumulative_buckets():
    from packmla.utils.metrics import LATENCY_BUCKETS, Metrics

    m = Metrics()
    for v in (0.003, 0.02, 0.02, 7.0, 1000.0):
        m.observe("ttft", v)
    h = m.histogram("ttft")
    assert h["count"] == 5 and abs(h["sum"] - 1007.043) < 1e-9
    assert h["buckets"]["0.005"] == 1 and h["buckets"]["0.025"] == 3 and h["buckets"]["10.0"] == 4
    assert h["buckets"]["+Inf"] == 5 and len(h["buckets"]) == len(LATENCY_BUCKETS) + 1
    text = m.prometheus()
    assert 'packmla_ttft_bucket{le="+Inf"} 5' in text and "packmla_ttft_count 5" in text
    assert "# TYPE packmla_ttft histogram" in text


def test_clients_send_the_api_key_from_the_environment(monkeypatch):
    from packmla.bench.serving import auth_headers

    monkeypatch.delenv("OPENAI_API_KEY", raising=False)
    monkeypatch.delenv("PACKMLA_API_KEY", raising=False)
    assert auth_headers() == {}
    monkeypatch.setenv("OPENAI_API_KEY", "k1")
    assert auth_headers() == {"Authorization": "Bearer k1"}
    monkeypatch.setenv("PACKMLA_API_KEY", "k2")
    assert auth_headers() == {"Authorization": "Bearer k2"}


def test_bench_phase_runs_every_request_to_its_length():
    """bench.py's serving phase on the tiny CPU model: all requests finish with their full output, the
    engine never runs more than C of them, and prompt chunks are counted as host -> device bytes."""
    import importlib.util
    import os

    import torch

    from packmla.config import EngineConfig, ModelConfig
    from packmla.engine.engine import Engine, SamplingParams
    from packmla.parallel.comm import TPComm

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_main", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = ModelConfig.tiny()
    C = 2
    eng = Engine.build(cfg, EngineConfig(max_running_requests=C, chunked_prefill_size=16, prefix_cache=True,
                                         disable_cuda_graph=True), "cpu", max_context=128, max_requests=C)
    running_max = []
    step = eng.step

    def watched():
        out = step()
        running_max.append(len(eng.running))
        return out

    eng.step = watched
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist() for _ in range(3 * C)]
    st = bench.run_phase(eng, prompts, SamplingParams(max_new_tokens=5), TPComm(), torch.device("cpu"), timed=True)
    assert st["out_tokens"] == 3 * C * 5
    assert max(running_max) <= C
    assert st["h2d"] >= 3 * C * 40 * 8  # every prompt token crossed as an int64
    assert st["wall_s"] > 0 and st["engine_steps"] >= 3 * C * 4
    eng.flush_cache()
    assert not eng.retained


def test_step_breakdown_groups_kernels_into_families():
    from packmla.bench.step_breakdown import family

    assert family("void (anonymous namespace)::mx_expert_kernel<0, 16>(CUtensorMap_st)") == "MoE experts (MXFP4)"
    assert family("(anonymous namespace)::moe_gather_slots_kernel(int const*)") == "MoE experts (MXFP4)"
    assert family("(anonymous namespace)::sparse_mla_decode_kernel(DecodeParams)") == "attention (sparse MLA decode)"
    assert family("(anonymous namespace)::index_logits_kernel(LogitParams)") == "indexer"
    assert family("nvjet_tst_32x64_64x16_4x1_v_bz_TNN") == "dense GEMM (cuBLAS)"
    assert family("void (anonymous namespace)::dense_mx_kernel<true>(CUtensorMap_st)") == \
        "dense projections, MXFP8 (packmla)"
    assert family("void at::native::vectorized_elementwise_kernel<4>") == "sampling / torch elementwise"
    assert family("something_else") == "other"


def test_engine_graph_buckets_end_at_the_concurrency():
    from packmla.bench.engine_setup import DEFAULT_CONCURRENCY, graph_buckets

    assert graph_buckets(8) == [1, 2, 4, 8]
    assert graph_buckets(40) == [1, 2, 4, 8, 16, 24, 32, 40]
    assert graph_buckets(5) == [1, 2, 4, 5]
    assert DEFAULT_CONCURRENCY == {1: 8, 2: 8, 4: 24, 8: 40}

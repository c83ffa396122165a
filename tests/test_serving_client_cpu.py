"""CPU: the serving benchmark client against a live packmla HTTP server (tiny model, HiCache on)."""
import json
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


def test_replay_of_recorded_sessions(server_url, tmp_path):
    from packmla.bench import replay

    url, eng = server_url
    path = tmp_path / "sessions.jsonl"
    with open(path, "w") as f:
        for s in range(3):
            history = [{"role": "user", "content": f"session {s} opening"}]
            for turn in range(2):
                f.write(json.dumps({"session": f"s{s}", "turn": turn, "messages": history, "max_tokens": 3}) + "\n")
                history = history + [{"role": "assistant", "content": "ok"}, {"role": "user", "content": "more"}]
    out = replay.main(["--base-url", url, "--requests", str(path), "--users", "2"])
    assert out["sessions"] == 3 and out["requests"] == 6 and out["success_rate"] == 1.0 and out["passed"]
    assert out["output_tokens"] >= 6 and out["ttft_ms"]["p50"] is not None
    sessions = replay.load_sessions(str(path))
    assert [[t["turn"] for t in s] for s in sessions] == [[0, 1]] * 3


def test_replay_sweep_ladder_and_stop(server_url, tmp_path):
    import csv

    from packmla.bench import replay

    url, eng = server_url
    path = tmp_path / "sessions.jsonl"
    with open(path, "w") as f:
        for s in range(3):
            f.write(json.dumps({"session": f"s{s}", "turn": 0, "max_tokens": 2,
                                "messages": [{"role": "user", "content": f"sweep {s}"}]}) + "\n")
    out = replay.main(["sweep", "--base-url", url, "--requests", str(path), "--concurrencies", "1,2",
                       "--repeats", "2", "--out-dir", str(tmp_path / "sw"), "--min-success", "1.0"])
    assert out["operational_complete"] and out["points"] == 4
    for c in (1, 2):
        for r in (1, 2):
            point = json.loads((tmp_path / "sw" / f"c{c}" / f"repeat-{r:02d}" / "summary.json").read_text())
            assert point["users"] == c and point["complete"] and point["ttft_ms"]["p90"] is not None
    rows = list(csv.DictReader(open(tmp_path / "sw" / "summary.csv")))
    assert [(r["concurrency"], r["repeat"]) for r in rows] == [("1", "1"), ("1", "2"), ("2", "1"), ("2", "2")]
    assert json.loads((tmp_path / "sw" / "manifest.json").read_text())["concurrencies"] == [1, 2]
    # a zero dispatch window starts no session; the gates report it
    win = replay.replay(url, str(path), 2, duration_s=0.0)
    assert win["sessions_started"] == 0 and win["requests"] == 0 and not win["passed"]
    # an unreachable server stops the sweep before its first point
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        dead = f"http://127.0.0.1:{s.getsockname()[1]}"
    res = replay.sweep(dead, str(path), [1], str(tmp_path / "sw2"))
    assert res["points"] == 0 and "unhealthy" in res["stopped"] and not res["operational_complete"]
    with pytest.raises(ValueError):
        replay.sweep(url, str(path), [2, 1], str(tmp_path / "sw3"))


def test_replay_capacity_plan(tmp_path):
    from packmla.bench import replay

    path = tmp_path / "plan.jsonl"
    sizes = {"s0": [10, 20], "s1": [5], "s2": [7, 7, 7]}
    with open(path, "w") as f:
        for sid, turns in sizes.items():
            for t, n in enumerate(turns):
                f.write(json.dumps({"session": sid, "turn": t, "messages": [], "prompt_tokens": n,
                                    "max_tokens": 0}) + "\n")
    out = replay.main(["plan", "--requests", str(path), "--concurrencies", "1,2,3", "--pool-tokens", "25"])
    peaks = {p["concurrency"]: p["peak_live_tokens"] for p in out["points"]}
    assert peaks == {1: 20, 2: 27, 3: 27}
    assert out["largest_fitting_concurrency"] == 1
    sessions = replay.load_sessions(str(path))
    assert replay.peak_live_tokens(sessions, 2, ticks=1) == 15
    assert replay.request_tokens({"messages": [{"content": "abc"}], "max_tokens": 4}) == 7


def test_request_slot_fifo_replay(server_url, tmp_path):
    from packmla.bench import replay

    url, eng = server_url
    path = tmp_path / "slots.jsonl"
    with open(path, "w") as f:
        for s in range(4):
            for t in range(2):
                f.write(json.dumps({"session": f"s{s}", "turn": t, "max_tokens": 2,
                                    "messages": [{"role": "user", "content": f"slot {s}/{t}"}]}) + "\n")
    out = replay.main(["--base-url", url, "--requests", str(path), "--scheduler", "request-slot", "--users", "2",
                       "--population", "3", "--duration-s", "120", "--min-success", "1.0"])
    assert out["finished"] == 8 and out["unresolved"] == 0 and out["completed_in_window"] == 8
    assert out["slo"]["status"] == "pass" and out["passed"]
    assert out["client_queue_ms"]["p50"] >= 0
    with pytest.raises(ValueError):
        replay.request_slot_replay(url, str(path), 3, 2, 10.0)  # population below concurrency
    assert replay.slo_status(9, 0, 10) == "pass"
    assert replay.slo_status(8, 0, 10) == "fail"
    assert replay.slo_status(8, 1, 10) == "indeterminate"


def test_auto_concurrency_from_the_server_pool(server_url):
    import requests

    from packmla.bench.serving import resolve_concurrency

    url, eng = server_url
    info = requests.get(url + "/server_info", timeout=30).json()
    assert info["context_length"] == eng.pool.max_context
    assert resolve_concurrency("auto", info, 100, 28) == info["max_total_num_tokens"] // 128
    assert resolve_concurrency("3", info, 100, 28) == 3
    with pytest.raises(SystemExit):  # longer than the server's context
        resolve_concurrency("1", info, info["context_length"], 1)
    with pytest.raises(SystemExit):  # the pool cannot hold one request
        resolve_concurrency("auto", {"max_total_num_tokens": 10}, 100, 28)


def test_convert_recorded_traffic(tmp_path):
    from packmla.bench import convert, replay

    raw = tmp_path / "raw.jsonl"
    recs = [
        {"id": "b2", "token_name": "u2", "created": 5.0, "messages": [{"role": "user", "content": "b second"}],
         "usage": {"prompt_tokens": 40, "completion_tokens": 7}},
        {"id": "a1", "token_name": "u1", "created": 1.0, "messages": [{"role": "user", "content": "a first"}],
         "usage": {"prompt_tokens": 10, "completion_tokens": 3}, "tools": [{"type": "function"}]},
        {"id": "b1", "token_name": "u2", "created": 2.0, "messages": [{"role": "user", "content": "b first"}],
         "usage": {"prompt_tokens": 20}},
        {"id": "solo", "created": 3.0, "messages": [{"role": "user", "content": "alone"}], "usage": {}},
    ]
    raw.write_text("\n".join(json.dumps(r) for r in recs) + "\n\n")
    out = convert.main(["--input", str(raw), "--output-dir", str(tmp_path / "prep")])
    assert out == {"output_dir": str((tmp_path / "prep").resolve()), "requests": 4, "sessions": 3}
    sessions = replay.load_sessions(str(tmp_path / "prep" / "sessions.jsonl"))
    assert [[t["request_id"] for t in s] for s in sessions] == [["a1"], ["b1", "b2"], ["solo"]]
    assert [t["turn"] for t in sessions[1]] == [0, 1]
    assert sessions[1][0]["max_tokens"] == 256 and sessions[1][1]["max_tokens"] == 7  # default cap when unrecorded
    assert sessions[0][0]["tools"] == [{"type": "function"}] and sessions[0][0]["ignore_eos"] is False
    lines = (tmp_path / "prep" / "requests.jsonl").read_text().splitlines()
    assert [json.loads(x)["request_id"] for x in lines] == ["b2", "a1", "b1", "solo"]  # source order
    man = json.loads((tmp_path / "prep" / "manifest.json").read_text())
    assert man["requests"] == 4 and [e["used_default_output_cap"] for e in man["records"]] == [False, False, True, True]
    # tick 0: a1 (10 + 3) and b1 (20 + 256); tick 1: b2 (40 + 7) and solo (5 content bytes + 256)
    assert replay.peak_live_tokens(sessions, 2) == max(13 + 276, 47 + 261)
    for bad, msg in ((dict(recs[1], id="b2"), "duplicate"), (dict(recs[1], created=float("nan")), "created"),
                     (dict(recs[1], messages=[]), "messages"), (dict(recs[1], usage=None), "usage")):
        p = tmp_path / "bad.jsonl"
        p.write_text(json.dumps(recs[0]) + "\n" + json.dumps(bad) + "\n")
        with pytest.raises(ValueError, match=msg):
            convert.convert(str(p), str(tmp_path / f"o-{msg}"))
        assert not (tmp_path / f"o-{msg}").exists()
    with pytest.raises(ValueError, match="exists"):
        convert.convert(str(raw), str(tmp_path / "prep"))


def test_client_disconnect_aborts_the_request(server_url):
    import asyncio

    import aiohttp

    url, eng = server_url
    before = eng.metrics.snapshot().get("requests_aborted", 0)

    async def go():
        async with aiohttp.ClientSession() as http:
            body = {"model": "tiny", "prompt": "abandon me", "max_tokens": 600, "stream": True, "ignore_eos": True}
            async with http.post(url + "/v1/completions", json=body) as resp:
                assert resp.status == 200
                async for raw in resp.content:
                    if raw.startswith(b"data: {"):
                        break  # one token seen; leave without reading the rest

    asyncio.run(go())
    deadline = time.time() + 30
    while time.time() < deadline:
        if eng.metrics.snapshot().get("requests_aborted", 0) > before and not eng.running and not eng.waiting:
            break
        time.sleep(0.05)
    assert eng.metrics.snapshot().get("requests_aborted", 0) == before + 1
    assert not eng.running and not eng.waiting


def test_serving_cli_writes_validated_wave_records(server_url, tmp_path):
    from packmla.bench import serving

    url, eng = server_url
    path = tmp_path / "waves.jsonl"
    serving.main(["--base-url", url, "--input-len", "50", "--output-len", "3", "--concurrency", "2",
                  "--output-file", str(path)])
    recs = [json.loads(x) for x in path.read_text().splitlines()]
    assert [r["phase"] for r in recs] == ["warmup", "measured"]
    assert recs[1]["completed"] == 6 and recs[1]["output_lens"] == [3] * 6 and recs[1]["validated"]
    with pytest.raises(FileExistsError):  # records are never overwritten
        serving.write_records(str(path), {"dataset": "random", "concurrency": 1, "input_len": 1, "output_len": 1})
    with pytest.raises(SystemExit, match="context"):  # longer than the server's context: refused up front
        serving.main(["--base-url", url, "--input-len", str(eng.pool.max_context), "--output-len", "3"])
    # a short response makes its wave invalid
    bad = serving.summarize([serving.Result(True, 5, [1, 2, 3]), serving.Result(False, 5, [1], error="short")], 1.0)
    assert not bad["validated"] and bad["output_lens"] == [3, 1]


def test_usage_reports_cached_prompt_tokens(server_url):
    import requests

    url, eng = server_url
    requests.post(url + "/flush_cache", timeout=30)
    p1 = [100 + (i * 7) % 200 for i in range(150)]
    r1 = requests.post(url + "/v1/completions", json={"model": "tiny", "prompt": p1, "max_tokens": 4,
                                                       "ignore_eos": True}, timeout=120).json()
    assert r1["usage"]["prompt_tokens_details"]["cached_tokens"] == 0
    out1 = r1["choices"][0]["token_ids"]
    p2 = p1 + out1 + [50, 51, 52]
    r2 = requests.post(url + "/v1/completions", json={"model": "tiny", "prompt": p2, "max_tokens": 2,
                                                       "ignore_eos": True}, timeout=120).json()
    assert r2["usage"]["prompt_tokens_details"]["cached_tokens"] == len(p1) + len(out1) - 1
    g = requests.post(url + "/generate", json={"input_ids": p2 + r2["choices"][0]["token_ids"] + [9],
                                               "sampling_params": {"max_new_tokens": 1, "ignore_eos": True}},
                      timeout=120).json()
    assert g["meta_info"]["cached_tokens"] == len(p2) + 1

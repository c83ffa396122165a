"""CPU: the environment-driven launcher (reference serve.sh / launch-config.sh names) resolves the
server command, owns the server's process group, waits for health and reads the pool out."""
import json
import os
import socket

import pytest

from packmla.server import launch


def test_env_names_map_onto_server_flags(tmp_path):
    env = {"MODE": "native", "TP": "4", "EP": "4", "PORT": "31000", "MASTER_PORT": "29700", "MEM_FRAC": "0.85",
           "CTX_LEN": "65536", "MAX_RUN": "40", "CHUNK": "4096", "SERVER_SEED": "42", "HICACHE_RATIO": "2",
           "DECODE_CFG": '{"decode": {"bs": [1, 2]}}', "C4_KEEP_COUNT": "256",
           "REQUEST_METRICS_DIR": str(tmp_path)}
    cmd, extra = launch.resolve(None, env)
    assert cmd[1:3] == ["-m", "torch.distributed.run"] and "--nproc-per-node" in cmd
    assert cmd[cmd.index("--nproc-per-node") + 1] == "4" and cmd[cmd.index("--master-addr") + 1] == "127.0.0.1"
    assert cmd[cmd.index("--master-port") + 1] == "29700"
    i = cmd.index("packmla.server")
    from packmla.server.__main__ import build_parser, resolve_args

    args = build_parser().parse_args(cmd[i + 1:])
    kw = resolve_args(args)
    assert args.tp == 4 and args.ep == 4 and args.port == 31000 and args.seed == 42 and args.context_length == 65536
    assert kw["kv_cache_format"] == "native" and kw["cuda_graph_bs"] == [1, 2]
    assert args.enable_hierarchical_cache and args.hicache_ratio == 2.0 and args.log_requests
    assert args.export_metrics_to_file_dir == str(tmp_path) and extra["NCCL_SOCKET_IFNAME"] == "lo"
    cmd1, _ = launch.resolve("direct", {"MODE": "native"})  # the positional mode wins; TP=1 runs directly
    assert cmd1[1:3] == ["-m", "packmla.server"] and cmd1[cmd1.index("--kv-cache-format") + 1] == "direct"
    with pytest.raises(SystemExit):
        launch.resolve(None, {"REQUEST_METRICS_DIR": str(tmp_path / "missing")})


def test_smoke_start_wait_readout_stop(monkeypatch, tmp_path, capsys):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    for k, v in {"MODEL": "tiny", "DEVICE": "cpu", "PORT": str(port), "MAX_RUN": "4", "CTX_LEN": "2048"}.items():
        monkeypatch.setenv(k, v)
    for k in ("TP", "WORLD_SIZE", "RANK", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        monkeypatch.delenv(k, raising=False)
    out = launch.main(["direct", "--smoke", "--wait-timeout", "300", "--log", str(tmp_path / "server.log")])
    assert out["event"] == "ready" and out["kv_cache_format"] == "direct" and out["max_total_num_tokens"] > 0
    assert out["prefix_cache"] is True and out["context_length"] == 2048
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["pgid"] == out["pgid"]
    with pytest.raises(ProcessLookupError):  # the whole group is gone
        os.killpg(out["pgid"], 0)


def test_sweep_owns_its_server(monkeypatch, tmp_path):
    import requests

    from packmla.bench import replay

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    for k, v in {"MODEL": "tiny", "DEVICE": "cpu", "PORT": str(port), "MAX_RUN": "4", "CTX_LEN": "2048"}.items():
        monkeypatch.setenv(k, v)
    for k in ("TP", "WORLD_SIZE", "RANK", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        monkeypatch.delenv(k, raising=False)
    path = tmp_path / "s.jsonl"
    path.write_text("".join(json.dumps({"session": f"s{i}", "turn": 0, "max_tokens": 2,
                                        "messages": [{"role": "user", "content": f"owned {i}"}]}) + "\n"
                            for i in range(2)))
    out = replay.main(["sweep", "--launch", "native", "--requests", str(path), "--concurrencies", "1,2",
                       "--out-dir", str(tmp_path / "sw"), "--min-success", "1.0", "--startup-timeout", "300"])
    assert out["operational_complete"] and out["points"] == 2 and out["server"]["kv_cache_format"] == "native"
    assert (tmp_path / "sw.server.log").exists()
    with pytest.raises(requests.RequestException):  # the owned server is gone
        requests.get(f"http://127.0.0.1:{port}/health", timeout=2)


def test_nsys_output_wraps_the_server(tmp_path):
    fake = tmp_path / "bin"
    fake.mkdir()
    (fake / "nsys").write_text("#!/bin/sh\nexit 0\n")
    (fake / "nsys").chmod(0o755)
    cmd, _ = launch.resolve("direct", {"NSYS_OUTPUT": str(tmp_path / "trace"), "PATH": str(fake)})
    assert cmd[0] == str(fake / "nsys") and "--capture-range=cudaProfilerApi" in cmd
    assert cmd[cmd.index("-o") + 1] == str(tmp_path / "trace") and "packmla.server" in cmd
    with pytest.raises(SystemExit, match="nsys"):
        launch.resolve("direct", {"NSYS_OUTPUT": "x", "PATH": str(tmp_path / "empty")})


def test_capacity_stress_compares_reuse_tiers(monkeypatch, tmp_path):
    from packmla.bench import capacity_stress

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    for k, v in {"MODEL": "tiny", "DEVICE": "cpu", "PORT": str(port), "MAX_RUN": "4", "CTX_LEN": "1024"}.items():
        monkeypatch.setenv(k, v)
    for k in ("TP", "WORLD_SIZE", "RANK", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT", "HICACHE_RATIO"):
        monkeypatch.delenv(k, raising=False)
    out = capacity_stress.main(["direct", "--settings", "none,prefix,hicache", "--sessions", "2", "--turns", "2",
                                "--input-len", "64", "--output-len", "4", "--concurrency", "2",
                                "--startup-timeout", "300", "--log-dir", str(tmp_path)])
    r = {x["setting"]: x for x in out["results"]}
    assert all(t["validated"] for x in r.values() for t in x["turns"])
    assert r["none"]["prefix_cache_hit_tokens"] == 0 and r["none"]["hicache_hit_tokens"] == 0
    assert r["prefix"]["prefix_cache_hit_tokens"] > 0 and r["prefix"]["hicache_hit_tokens"] == 0
    assert r["hicache"]["hicache_hit_tokens"] > 0 and r["hicache"]["prefix_cache_hit_tokens"] == 0
    # reuse means less prefill work for the same conversation
    assert r["prefix"]["prefill_tokens"] < r["none"]["prefill_tokens"]
    assert r["hicache"]["prefill_tokens"] < r["none"]["prefill_tokens"]


def test_model_families_are_validated_like_the_reference_launcher():
    import pytest

    from packmla.server.launch import resolve

    cmd, _ = resolve("direct", {"MODEL_FAMILY": "dsv41", "TP": "4"})
    assert cmd[cmd.index("--kv-cache-format") + 1] == "fp4-direct" and cmd[cmd.index("--ep") + 1] == "4"
    cmd, _ = resolve("native", {"MODEL_FAMILY": "dsv41", "TP": "2", "GPUS": "0,1"})
    assert cmd[cmd.index("--kv-cache-format") + 1] == "fp4-native" and cmd[cmd.index("--tp") + 1] == "2"
    for env, msg in (({"MODEL_FAMILY": "dsv41", "TP": "3"}, "1, 2, 4 or 8"),
                     ({"MODEL_FAMILY": "dsv41", "TP": "4", "EP": "3"}, "does not divide"),
                     ({"MODEL_FAMILY": "dsv41", "TP": "2", "EP": "1"}, "EP = TP"),
                     ({"MODEL_FAMILY": "dsv41", "HICACHE_RATIO": "2"}, "HiCache"),
                     ({"MODEL_FAMILY": "dsv41", "TP": "2", "GPUS": "0,"}, "exactly 2 devices"),
                     ({"MODEL_FAMILY": "glm53", "C4_KEEP_COUNT": "128"}, "dsv4 only"),
                     ({"MODEL_FAMILY": "glm53"}, "not built"),
                     ({"MODEL_FAMILY": "glm99"}, "unknown MODEL_FAMILY")):
        with pytest.raises(SystemExit, match=msg):
            resolve("direct", env)
    cmd, _ = resolve("direct", {})
    assert cmd[cmd.index("--kv-cache-format") + 1] == "direct"
    assert cmd[cmd.index("--reasoning-parser") + 1] == "deepseek-v4"


def test_frontend_preparation_and_diagnostics_environment():
    import pytest

    from packmla.server.launch import resolve

    cmd, _ = resolve("direct", {"DSV4_ASYNC_PREPARATION": "1", "DSV4_PREPARATION_WORKERS": "4",
                                "FRONTEND_DIAGNOSTICS": "1"})
    assert cmd[cmd.index("--chat-preparation-workers") + 1] == "4" and "--frontend-diagnostics" in cmd
    cmd, _ = resolve("direct", {})
    assert "--chat-preparation-workers" not in cmd and "--frontend-diagnostics" not in cmd
    for env, msg in (({"DSV4_PREPARATION_WORKERS": "3"}, "takes 1, 2 or 4"), ({"FRONTEND_DIAGNOSTICS": "yes"}, "takes 0 or 1"),
                     ({"DSV4_ASYNC_PREPARATION": "2"}, "takes 0 or 1")):
        with pytest.raises(SystemExit, match=msg):
            resolve("native", env)
    from packmla.server.__main__ import build_parser

    a = build_parser().parse_args(["--chat-preparation-workers", "2", "--frontend-diagnostics"])
    assert a.chat_preparation_workers == 2 and a.frontend_diagnostics

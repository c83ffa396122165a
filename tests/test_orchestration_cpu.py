"""CPU: host orchestration tools (environment helpers, kernel runner, qualification receipts, serving runner,
capture launcher, container image definition)."""
import http.server
import json
import socket
import subprocess
import sys
import threading
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_env_report_health_pool_and_kill_port():
    from packmla.utils import env

    rep = env.report()
    assert "environment" in rep and isinstance(rep["gpus"], list) and "nccl_env" in rep

    class H(http.server.BaseHTTPRequestHandler):
        def do_GET(self):
            body = b"ok" if self.path == "/health" else json.dumps({"max_total_num_tokens": 4096, "tp": 1}).encode()
            self.send_response(200)
            self.end_headers()
            self.wfile.write(body)

        def log_message(self, *a):
            pass

    srv = http.server.HTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    url = f"http://127.0.0.1:{srv.server_port}"
    try:
        assert env.health(url) and env.pool_of(url) == {"max_total_num_tokens": 4096, "tp": 1}
    finally:
        srv.shutdown()
    assert not env.health(f"http://127.0.0.1:{_free_port()}")
    port = _free_port()
    child = subprocess.Popen([sys.executable, "-c", f"import socket,time;s=socket.socket();"
                              f"s.bind(('127.0.0.1',{port}));s.listen();time.sleep(60)"])
    try:
        for _ in range(100):
            if env.listener_pid(port):
                break
            time.sleep(0.05)
        assert env.kill_port(port, grace_s=5) == child.pid
        assert child.wait(5) is not None
    finally:
        if child.poll() is None:
            child.kill()


def test_kernel_runner_is_fail_closed_and_sealed(tmp_path):
    from packmla.bench import kernel_runner

    calls = []

    def fake(cmd, log, timeout):
        calls.append(cmd)
        with open(log, "a") as f:
            f.write("ran\n")
        return 1 if "validate" in str(log) else 0

    out = kernel_runner.run(tmp_path / "run", ["decode", "store"], ["validate", "bench"], execute=fake)
    names = [(r["stage"], r["status"]) for r in out["records"]]
    assert names[0] == ("validate.decode", "failed") and all(s == "skipped" for _, s in names[1:])
    assert not out["passed"] and len(calls) == 1
    assert (tmp_path / "run" / "SHA256SUMS").exists() and (tmp_path / "run" / "manifest.json").exists()
    with pytest.raises(ValueError, match="fresh"):
        kernel_runner.run(tmp_path / "run", ["decode"], ["bench"], execute=fake)
    prof = kernel_runner.profile_cmds("decode", tmp_path)
    assert prof[1][:5] == ["ncu", "--set", "full", "--clock-control", "none"] and "-c" in prof[1]


def _sealed(run_dir: Path, stages, bench_rows, identity=True):
    from packmla.utils.provenance import write_sums

    run_dir.mkdir()
    (run_dir / "manifest.json").write_text(json.dumps({"sources": {
        "library_matches_sources": identity, "compiled_modified": [], "csrc_sha256": "x"}}))
    (run_dir / "stages.json").write_text(json.dumps(stages))
    (run_dir / "bench.decode.log").write_text("\n".join(json.dumps(r) for r in bench_rows) + "\n")
    write_sums(run_dir)


def test_qualification_receipts(tmp_path):
    from packmla.bench import qualify

    good_clock = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    stages = [{"stage": "validate.decode", "status": "passed"}, {"stage": "bench.decode", "status": "passed"}]
    _sealed(tmp_path / "ok", stages, [{"case": "decode", "us": 20.0, "clocks": good_clock}])
    r = qualify.qualify(tmp_path / "ok", ["validate", "bench"])
    assert r["qualified"], r["checks"]
    assert r["notes"]  # sw_power_cap noted, not rejected
    assert qualify.main([str(tmp_path / "ok"), "--require", "validate,bench"]) == 0
    assert json.loads((tmp_path / "ok.qualification.json").read_text())["qualified"]
    # each failure alone rejects: a throttled clock, a skipped stage, a changed file, a foreign library
    _sealed(tmp_path / "hot", stages, [{"case": "decode", "clocks": {**good_clock, "reasons": ["hw_slowdown"]}}])
    assert not qualify.qualify(tmp_path / "hot", ["validate", "bench"])["qualified"]
    _sealed(tmp_path / "skip", stages[:1] + [{"stage": "bench.decode", "status": "skipped"}],
            [{"case": "decode", "clocks": good_clock}])
    assert not qualify.qualify(tmp_path / "skip", ["validate", "bench"])["qualified"]
    _sealed(tmp_path / "edit", stages, [{"case": "decode", "clocks": good_clock}])
    (tmp_path / "edit" / "bench.decode.log").write_text("{}\n")
    assert not qualify.qualify(tmp_path / "edit", ["validate", "bench"])["qualified"]
    _sealed(tmp_path / "lib", stages, [{"case": "decode", "clocks": good_clock}], identity=False)
    assert not qualify.qualify(tmp_path / "lib", ["validate", "bench"])["qualified"]
    assert not qualify.qualify(tmp_path / "missing", ["validate"])["qualified"]


def test_serving_runner_smoke_on_cpu(tmp_path):
    from packmla.bench import serve_runner

    env = {"MODEL": "tiny", "DEVICE": "cpu", "PORT": str(_free_port()), "MASTER_PORT": str(_free_port())}
    out = serve_runner.run(tmp_path / "serve", "direct", env, smoke_only=True, wait_timeout=300)
    steps = {s["step"]: s for s in out["steps"]}
    assert out["passed"], out["steps"]
    assert steps["launch"]["pool"]["kv_cache_format"] == "direct" and steps["smoke"]["passed"]
    assert "stop" in steps and (tmp_path / "serve" / "SHA256SUMS").exists()
    bad = serve_runner.run(tmp_path / "serve2", "direct", env, checkpoint=tmp_path, profile="dsv4",
                           smoke_only=True)
    assert not bad["passed"] and [s["step"] for s in bad["steps"]] == ["checkpoint"]


def test_capture_launcher_deadline_failure_and_success(tmp_path):
    from packmla.training.data import capture_launch

    py = sys.executable
    out = tmp_path / "cache"
    slow = [py, "-c", "import os,sys,time; os.makedirs(sys.argv[1]); time.sleep(60)", "{output}"]
    rec = capture_launch.launch(["--output", str(out)], deadline_s=1.0, grace_s=5.0, command=slow)
    assert rec["outcome"] == "deadline" and not out.exists()
    assert not list(tmp_path.glob("cache.staging-*"))  # the partial output was removed
    failing = [py, "-c", "import os,sys; os.makedirs(sys.argv[1]); sys.exit(3)", "{output}"]
    rec = capture_launch.launch(["--output", str(out)], deadline_s=30.0, command=failing)
    assert rec["outcome"] == "failed" and rec["exit_code"] == 3 and not out.exists()
    good = [py, "-c", "import os,sys; os.makedirs(sys.argv[1]); open(sys.argv[1] + '/index.json', 'w').write('{}')",
            "{output}"]
    rec = capture_launch.launch(["--output", str(out)], deadline_s=30.0, command=good)
    assert rec["outcome"] == "completed" and (out / "index.json").exists()
    assert json.loads((tmp_path / "cache.launch.json").read_text())["outcome"] == "completed"
    with pytest.raises(ValueError, match="fresh"):
        capture_launch.launch(["--output", str(out)], deadline_s=1.0, command=good)


def test_image_definition_builds_and_gates_the_extension():
    text = (ROOT / "docker" / "Dockerfile").read_text()
    assert "python setup.py build_ext --inplace" in text and "packmla.utils.provenance sources" in text
    assert "nvidia/cuda:12.9" in text and "packmla.server" in text

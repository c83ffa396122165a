"""CPU: `python -m packmla.server` starts, serves the OpenAI routes and shuts down (tiny model)."""
import json
import os
import signal
import socket
import subprocess
import sys
import time

import requests

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_server_process_end_to_end():
    port = _free_port()
    # launched with the reference launcher's flag names
    proc = subprocess.Popen([sys.executable, "-m", "packmla.server", "--model-path", "tiny", "--device", "cpu",
                             "--port", str(port), "--max-running-requests", "4", "--context-length", "1024",
                             "--kv-cache-format", "direct", "--kv-cache-dtype", "fp8_e4m3", "--random-seed", "3",
                             "--watchdog-timeout", "600", "--enable-hierarchical-cache", "--hicache-ratio", "2.0",
                             "--hicache-write-policy", "write_through", "--enable-metrics"],
                            cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                            start_new_session=True)
    url = f"http://127.0.0.1:{port}"
    try:
        for _ in range(600):
            try:
                if requests.get(url + "/health", timeout=1).text == "ok":
                    break
            except requests.RequestException:
                pass
            if proc.poll() is not None:
                raise AssertionError(f"server exited early: {proc.stdout.read()}")
            time.sleep(0.2)
        info = requests.get(url + "/server_info", timeout=10).json()
        assert info["kv_cache_format"] == "direct" and info["enable_hierarchical_cache"]
        r = requests.post(url + "/v1/completions", json={"prompt": "hello", "max_tokens": 3, "ignore_eos": True},
                          timeout=60).json()
        assert len(r["choices"][0]["token_ids"]) == 3
        c = requests.post(url + "/v1/chat/completions", timeout=60,
                          json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 2,
                                "ignore_eos": True}).json()
        assert c["usage"]["completion_tokens"] == 2
        assert "packmla_requests_finished" in requests.get(url + "/metrics", timeout=10).text
    finally:
        os.killpg(proc.pid, signal.SIGTERM)  # the server's own process group
        try:
            proc.wait(30)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)
            proc.wait(30)

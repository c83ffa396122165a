"""Per-request logging and metric export of the server.

Reference behaviour: the reference launches SGLang with `--enable-metrics --log-requests
--export-metrics-to-file` (scripts/local/run-server.sh:150-154): every finished request is logged,
and its timing metrics are appended to files under a directory for later joins with the client's
records.  `RequestLogger` receives one record per finished request from the engine driver:

    {"time": unix seconds, "id": request id, "prompt_tokens": P, "completion_tokens": N,
     "finish_reason": "length" | "stop" | "abort" | "error", "ttft_s": ..., "e2e_s": ..., "tpot_s": ...}

`log_level` (--log-requests-level) adds 1: sampling parameters, 2: the first 64 output token ids,
3: every prompt and output token id.  With `export_dir`, records are appended as JSON lines to
`<export_dir>/request-metrics-<YYYYmmdd_HH>.jsonl` (one file per UTC hour).
"""
from __future__ import annotations

import json
import logging
import os
import threading
import time
from dataclasses import asdict

log = logging.getLogger("packmla.requests")


class RequestLogger:
    def __init__(self, log_requests: bool = False, log_level: int = 0, export_dir: str | None = None):
        if not 0 <= log_level <= 3:
            raise ValueError("--log-requests-level is 0..3")
        self.log_requests = log_requests
        self.log_level = log_level
        self.export_dir = export_dir
        self._lock = threading.Lock()
        if export_dir:
            os.makedirs(export_dir, exist_ok=True)

    @property
    def enabled(self) -> bool:
        return self.log_requests or bool(self.export_dir)

    def record(self, st, prompt: list[int] | None = None) -> dict:
        """The record of a finished driver `Stream`."""
        now = time.perf_counter()
        n = len(st.tokens)
        ttft = None if st.t_first is None else st.t_first - st.t_submit
        rec = {"time": time.time(), "id": st.ext_id, "prompt_tokens": st.prompt_len, "completion_tokens": n,
               "finish_reason": st.finish_reason, "ttft_s": ttft, "e2e_s": now - st.t_submit,
               "tpot_s": (now - st.t_first) / (n - 1) if st.t_first is not None and n > 1 else None}
        if self.log_level >= 1 and st.params is not None:
            rec["sampling_params"] = asdict(st.params)
        if self.log_level == 2:
            rec["output_ids"] = list(st.tokens[:64])
        if self.log_level >= 3:
            rec["output_ids"] = list(st.tokens)
            rec["prompt_ids"] = list(prompt) if prompt is not None else None
        return rec

    def finished(self, st, prompt: list[int] | None = None) -> None:
        if not self.enabled:
            return
        rec = self.record(st, prompt)
        line = json.dumps(rec)
        if self.log_requests:
            log.info("request finished %s", line)
        if self.export_dir:
            name = time.strftime("request-metrics-%Y%m%d_%H.jsonl", time.gmtime(rec["time"]))
            with self._lock, open(os.path.join(self.export_dir, name), "a") as f:
                f.write(line + "\n")

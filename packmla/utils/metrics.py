"""Prometheus-style counters for the engine (tokens, steps, pool occupancy, device time)."""
from __future__ import annotations

import threading
from collections import defaultdict


class Metrics:
    def __init__(self):
        self._c = defaultdict(float)
        self._lock = threading.Lock()

    def inc(self, name: str, v: float = 1.0) -> None:
        with self._lock:
            self._c[name] += v

    def set(self, name: str, v: float) -> None:
        with self._lock:
            self._c[name] = v

    def snapshot(self) -> dict:
        with self._lock:
            return dict(self._c)

    def prometheus(self, prefix: str = "packmla_") -> str:
        return "".join(f"{prefix}{k} {v}\n" for k, v in sorted(self.snapshot().items()))

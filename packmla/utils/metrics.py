"""Prometheus-style counters, gauges and latency histograms for the engine and server (tokens, steps,
pool occupancy, TTFT / end-to-end / per-token latency)."""
from __future__ import annotations

import threading
from collections import defaultdict


# latency buckets in seconds (upper bounds; +Inf is implicit), as fine as serving dashboards use
LATENCY_BUCKETS = (0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 25.0, 50.0, 100.0, 300.0)


class Metrics:
    def __init__(self):
        self._c = defaultdict(float)
        self._h: dict[str, list] = {}  # name -> [bucket counts..., +Inf count, sum]
        self._lock = threading.Lock()

    def observe(self, name: str, v: float, buckets=LATENCY_BUCKETS) -> None:
        """Add one observation to histogram `name` (cumulative buckets on export)."""
        with self._lock:
            h = self._h.setdefault(name, [0] * (len(buckets) + 1) + [0.0])
            i = next((j for j, b in enumerate(buckets) if v <= b), len(buckets))
            h[i] += 1
            h[-1] += v

    def histogram(self, name: str, buckets=LATENCY_BUCKETS) -> dict:
        with self._lock:
            h = list(self._h.get(name, [0] * (len(buckets) + 1) + [0.0]))
        cum, acc = [], 0
        for c in h[:-1]:
            acc += c
            cum.append(acc)
        return {"buckets": dict(zip([*map(str, buckets), "+Inf"], cum)), "count": acc, "sum": h[-1]}

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
        out = [f"{prefix}{k} {v}\n" for k, v in sorted(self.snapshot().items())]
        with self._lock:
            names = sorted(self._h)
        for name in names:
            h = self.histogram(name)
            out.append(f"# TYPE {prefix}{name} histogram\n")
            out += [f'{prefix}{name}_bucket{{le="{le}"}} {n}\n' for le, n in h["buckets"].items()]
            out += [f"{prefix}{name}_count {h['count']}\n", f"{prefix}{name}_sum {h['sum']}\n"]
        return "".join(out)

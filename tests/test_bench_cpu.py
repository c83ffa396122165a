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

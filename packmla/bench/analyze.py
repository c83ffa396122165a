"""Compare two sweep records point by point (for instance Native against Direct at the same ladder).

    python -m packmla.bench.analyze results/sweep-native results/sweep-direct [--output cmp.json]

Reads the `summary.json` of two `python -m packmla.bench.replay sweep` runs, pairs their points by
(concurrency, repeat), and reports per point the candidate / baseline ratio of successful requests/s,
output tokens/s and TTFT p90, with each side's gate results; then the geometric means of the ratios
over the points both sides completed.  Points present on one side only are listed, never dropped
silently.  Reference behaviour: the analysis scripts kept beside its replay records
(benchmarks/lswb-replay/.../analyze.py), which compare Native and Packed runs of the same protocol.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

METRICS = (("successful_requests_per_s", "higher"), ("output_throughput_tok_s", "higher"),
           ("ttft_p90_ms", "lower"))


def _points(run: Path) -> dict:
    data = json.loads((Path(run) / "summary.json").read_text())
    out = {}
    for p in data["points"]:
        out[(p["concurrency"], p["repeat"])] = {
            "successful_requests_per_s": p.get("successful_requests_per_s"),
            "output_throughput_tok_s": p.get("output_throughput_tok_s"),
            "ttft_p90_ms": (p.get("ttft_ms") or {}).get("p90"),
            "passed": p.get("passed"), "success_rate": p.get("success_rate")}
    return out


def _geomean(xs: list[float]) -> float | None:
    xs = [x for x in xs if x is not None and x > 0 and math.isfinite(x)]
    return math.exp(sum(math.log(x) for x in xs) / len(xs)) if xs else None


def compare(baseline: str, candidate: str) -> dict:
    a, b = _points(Path(baseline)), _points(Path(candidate))
    rows, ratios = [], {m: [] for m, _ in METRICS}
    for key in sorted(set(a) & set(b)):
        row = {"concurrency": key[0], "repeat": key[1], "baseline_passed": a[key]["passed"],
               "candidate_passed": b[key]["passed"]}
        for m, _ in METRICS:
            x, y = a[key][m], b[key][m]
            r = (y / x) if (x and y is not None) else None
            row[f"{m}_ratio"] = r
            ratios[m].append(r)
        rows.append(row)
    return {"baseline": str(baseline), "candidate": str(candidate), "points": rows,
            "geomean_ratio": {m: _geomean(ratios[m]) for m, _ in METRICS},
            "better_when": dict(METRICS),
            "only_baseline": sorted(list(k) for k in set(a) - set(b)),
            "only_candidate": sorted(list(k) for k in set(b) - set(a))}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("baseline")
    ap.add_argument("candidate")
    ap.add_argument("--output", default=None, help="also write the comparison here (a new file)")
    a = ap.parse_args(argv)
    out = compare(a.baseline, a.candidate)
    text = json.dumps(out, indent=2)
    if a.output:
        with open(a.output, "x") as f:
            f.write(text)
    print(text)
    return out


if __name__ == "__main__":
    main()

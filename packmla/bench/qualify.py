"""Qualification receipt of a sealed run directory (fail-closed).

    python -m packmla.bench.qualify RUN_DIR [--require build,validate,bench]

Reference behaviour: scripts/modal/qualification.py and kernel_qualification.py (receipt and identity
checks, fail-closed treatment of partial evidence).  A run qualifies only when every check passes:

  * integrity: the directory holds exactly the files its SHA256SUMS lists, with those hashes;
  * identity: the manifest records an extension built from the csrc/ it ran with, and no compiled source
    modified against the recorded commit;
  * stages: every required stage ran and passed (`stages.json` of packmla.bench.kernel_runner), none was
    skipped;
  * timing: every benchmark JSON line in the bench logs has a clock record without hardware or thermal
    slowdown and not stuck below 80 % of the maximum SM clock with no reason (`sw_power_cap` is noted);
  * profiles: each profile stage left its ncu report and metric export.

Missing evidence rejects the run.  The receipt is written beside the directory as
`<RUN_DIR>.qualification.json` (writing into the sealed directory would change its contents); the exit
code is 0 for a qualified run, 1 otherwise.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

BAD_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def _check_clock(row: dict, min_fraction: float = 0.8) -> str | None:
    clk = row.get("clocks") or {}
    reasons = clk.get("reasons") or []
    bad = [r for r in reasons if r in BAD_REASONS]
    if bad:
        return "clock slowdown: " + ", ".join(bad)
    if not clk.get("sm_mhz") or not clk.get("sm_max_mhz"):
        return "no clock record"
    if clk["sm_mhz"] < min_fraction * clk["sm_max_mhz"] and "sw_power_cap" not in reasons:
        return f"SM clock {clk['sm_mhz']} MHz well below max with no reason"
    return None


def qualify(run_dir: Path, require: list[str]) -> dict:
    from ..utils.provenance import verify_run

    run_dir = Path(run_dir)
    checks: list[dict] = []

    def check(name: str, ok: bool, detail=None):
        checks.append({"check": name, "ok": bool(ok), **({"detail": detail} if detail else {})})

    problems = verify_run(run_dir)
    check("integrity", not problems, problems or None)
    try:
        manifest = json.loads((run_dir / "manifest.json").read_text())
        src = manifest["sources"]
        check("identity: extension built from these sources", src.get("library_matches_sources") is True,
              {"csrc_sha256": src.get("csrc_sha256")})
        check("identity: compiled sources unmodified", not src.get("compiled_modified"), src.get("compiled_modified"))
    except (OSError, KeyError, ValueError) as exc:
        check("identity", False, f"manifest unreadable: {exc}")
    try:
        stages = json.loads((run_dir / "stages.json").read_text())
    except (OSError, ValueError) as exc:
        stages = []
        check("stages", False, f"stages.json unreadable: {exc}")
    for req in require:
        mine = [s for s in stages if s["stage"] == req or s["stage"].startswith(req + ".")]
        check(f"stage {req}", bool(mine) and all(s["status"] == "passed" for s in mine),
              [{"stage": s["stage"], "status": s["status"]} for s in mine] or "not run")
    notes = []
    bench_logs = sorted(run_dir.glob("bench*.log"))
    if "bench" in require:
        rows = 0
        bad = []
        for log in bench_logs:
            for line in log.read_text().splitlines():
                if not line.startswith("{"):
                    continue
                row = json.loads(line)
                rows += 1
                why = _check_clock(row)
                if why:
                    bad.append({"log": log.name, "case": row.get("case"), "reason": why})
                if "sw_power_cap" in ((row.get("clocks") or {}).get("reasons") or []):
                    notes.append({"log": log.name, "note": "sw_power_cap active"})
        check("timing records", rows > 0 and not bad, bad or ("no benchmark records" if rows == 0 else None))
    for s in stages:
        if s["stage"].startswith("profile.") and s["status"] == "passed":
            fam = s["stage"].split(".", 1)[1]
            have = (run_dir / f"profile.{fam}.ncu-rep").exists() and (run_dir / f"profile.{fam}.csv").exists()
            check(f"profile {fam}", have, None if have else "report or metric export missing")
    qualified = bool(checks) and all(c["ok"] for c in checks)
    return {"run_dir": str(run_dir), "qualified": qualified, "checks": checks, "notes": notes}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("run_dir", type=Path)
    ap.add_argument("--require", default="build,validate,bench")
    a = ap.parse_args(argv)
    receipt = qualify(a.run_dir, [x for x in a.require.split(",") if x])
    out = a.run_dir.with_name(a.run_dir.name + ".qualification.json")
    out.write_text(json.dumps(receipt, indent=1) + "\n")
    print(json.dumps({"qualified": receipt["qualified"], "receipt": str(out)}))
    return 0 if receipt["qualified"] else 1


if __name__ == "__main__":
    sys.exit(main())

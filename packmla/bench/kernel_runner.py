"""Kernel runner: build, validate, benchmark and profile kernel families into one sealed run directory.

    python -m packmla.bench.kernel_runner RUN_DIR [--families decode,store] [--stages build,validate,bench,profile]

Reference behaviour: scripts/modal/kernels.py (`prepare_kernels`, `preflight_kernels`, `validate_kernels`,
`benchmark_kernels`, `profile_kernels`: one image, the same stages in order, logs and receipts per run).
packmla runs the stages on the GPU host it is on:

  build     `setup.py build_ext --inplace` (sm_100a only), then the source gate (the extension must have
            been built from the csrc/ in the tree: packmla.utils.provenance);
  validate  `pytest -m gpu -x` over the family's test selection;
  bench     the family's microbenchmark cases, one JSON line each (decode cases with the reference's
            timing protocol), each with its clock record;
  profile   one small `ncu --set full --clock-control none` capture of the family's kernel (one launch),
            only after the same command has exited 0 without ncu; the capture's headline metrics are
            exported as CSV (`ncu -i ... --page raw --csv`) beside the report.

Each stage writes `<stage>[.<family>].log` and a record in `stages.json` (command, exit code, seconds).  A
failed stage stops the run, and later stages are recorded as skipped (fail-closed).  At the end the
directory is sealed (manifest.json + SHA256SUMS) for `packmla.bench.qualify`.  compute-sanitizer is not
part of the runner: device-side checks use the kernels' bounded waits and error word instead.
"""
from __future__ import annotations

import argparse
import json
import shlex
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
PY = sys.executable
MB = [PY, "-m", "packmla.bench.microbench"]

# family -> (pytest selection, microbenchmark cases, (kernel regex, small command for one capture))
FAMILIES: dict[str, dict] = {
    "decode": {
        "tests": ["tests/test_gpu_kernels.py", "-k", "decode", "tests/test_zz_no_alloc.py"],
        "bench": [MB + ["decode", "--batch", str(b), "--heads", str(h), "--topk", "512", "--swa", "128",
                        "--context", "32768", "--kv-format", f, "--protocol", "reference", "--rounds", "30"]
                  for b, h in ((8, 64), (16, 128)) for f in ("native", "direct")],
        "profile": ("sparse_mla_decode_kernel",
                    MB + ["decode", "--batch", "8", "--heads", "64", "--topk", "512", "--swa", "128", "--context",
                          "32768", "--kv-format", "direct", "--rounds", "1", "--warmup", "1"]),
    },
    "store": {
        "tests": ["tests/test_gpu_kernels.py", "-k", "store", "tests/test_gpu_adapter.py"],
        "bench": [MB + ["store", "--rows", str(r), "--kv-format", f] for r in (24, 8192) for f in ("native", "direct")],
        "profile": ("packed_store_kernel", MB + ["store", "--rows", "8192", "--kv-format", "direct", "--rounds", "1",
                                                 "--warmup", "1"]),
    },
    "moe": {
        "tests": ["tests/test_gpu_model.py", "-k", "moe or expert", "tests/test_gpu_blockscaled.py"],
        "bench": [MB + ["moe", "--tokens", str(t)] for t in (40, 512)],
        "profile": ("mx_expert_kernel", MB + ["moe", "--tokens", "40", "--rounds", "1", "--warmup", "1"]),
    },
    "dense": {
        "tests": ["tests/test_gpu_dense.py"],
        "bench": [MB + ["dense"]],
        "profile": ("dense_mx_kernel", MB + ["dense", "--rounds", "1", "--warmup", "1"]),
    },
    "indexer": {
        "tests": ["tests/test_gpu_indexer.py"],
        "bench": [MB + ["index"]],
        "profile": ("index", MB + ["index", "--rounds", "1", "--warmup", "1"]),
    },
    "fp4": {
        "tests": ["tests/test_gpu_kernels.py", "-k", "fp4"],
        "bench": [MB + ["fp4-suite", "--context", "32768", "--protocol", "reference"]],
        "profile": ("sparse_mla_decode_kernel",
                    MB + ["decode", "--batch", "8", "--heads", "64", "--topk", "512", "--swa", "128", "--context",
                          "32768", "--kv-format", "fp4-direct", "--rounds", "1", "--warmup", "1"]),
    },
    "glm": {  # GLM-5.3 rows: stores, Adapter and the decode row kinds (the reference's --model-family glm53)
        "tests": ["tests/test_gpu_glm.py"],
        "bench": [MB + ["glm-suite", "--rounds", "30"]],
        "profile": ("sparse_mla_decode_kernel",
                    MB + ["glm-suite", "--rounds", "1", "--warmup", "1", "--glm-batches", "8"]),
    },
}
STAGES = ("build", "validate", "bench", "profile")
NCU_METRICS = ("gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum",
               "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
               "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
               "sm__warps_active.avg.pct_of_peak_sustained_active", "launch__registers_per_thread")


class Runner:
    def __init__(self, run_dir: Path, execute=None):
        self.dir = Path(run_dir)
        self.records: list[dict] = []
        self.failed = False
        self._exec = execute or self._subprocess

    @staticmethod
    def _subprocess(cmd: list[str], log: Path, timeout: float) -> int:
        with open(log, "ab") as f:
            f.write(("$ " + shlex.join(cmd) + "\n").encode())
            f.flush()
            try:
                return subprocess.run(cmd, cwd=ROOT, stdout=f, stderr=subprocess.STDOUT, timeout=timeout).returncode
            except subprocess.TimeoutExpired:
                f.write(b"\n[runner] timed out\n")
                return 124

    def step(self, stage: str, family: str | None, cmds: list[list[str]], timeout: float = 3600.0) -> bool:
        name = stage if family is None else f"{stage}.{family}"
        if self.failed:
            self.records.append({"stage": name, "status": "skipped", "reason": "an earlier stage failed"})
            return False
        log = self.dir / f"{name}.log"
        t0 = time.time()
        rc = 0
        for cmd in cmds:
            rc = self._exec(cmd, log, timeout)
            if rc != 0:
                break
        rec = {"stage": name, "status": "passed" if rc == 0 else "failed", "exit_code": rc,
               "seconds": round(time.time() - t0, 1), "commands": [shlex.join(c) for c in cmds]}
        self.records.append(rec)
        self.failed = rc != 0
        return rc == 0

    def write(self) -> None:
        (self.dir / "stages.json").write_text(json.dumps(self.records, indent=1) + "\n")


def profile_cmds(family: str, run_dir: Path) -> list[list[str]]:
    """Plain run first (it must exit 0), then one capture of one launch, then the CSV export."""
    kernel, cmd = FAMILIES[family]["profile"]
    rep = str(run_dir / f"profile.{family}")
    return [cmd,
            ["ncu", "--set", "full", "--clock-control", "none", "-k", f"regex:{kernel}", "-c", "1", "-o", rep] + cmd,
            ["ncu", "-i", rep + ".ncu-rep", "--page", "raw", "--csv", "--metrics", ",".join(NCU_METRICS),
             "--log-file", str(run_dir / f"profile.{family}.csv")]]


def run(run_dir: Path, families: list[str], stages: list[str], execute=None, seal: bool = True) -> dict:
    run_dir = Path(run_dir)
    if run_dir.exists() and any(run_dir.iterdir()):
        raise ValueError(f"fresh run directory required: {run_dir}")
    run_dir.mkdir(parents=True, exist_ok=True)
    unknown = set(families) - set(FAMILIES) or set(stages) - set(STAGES)
    if unknown:
        raise ValueError(f"unknown families or stages: {sorted(unknown)}")
    r = Runner(run_dir, execute)
    if "build" in stages:
        r.step("build", None, [[PY, "setup.py", "build_ext", "--inplace"],
                               [PY, "-m", "packmla.utils.provenance", "sources"]])
    for fam in families:
        spec = FAMILIES[fam]
        if "validate" in stages:
            r.step("validate", fam, [[PY, "-m", "pytest", "-m", "gpu", "-x", "-q"] + spec["tests"]])
        if "bench" in stages:
            r.step("bench", fam, spec["bench"])
        if "profile" in stages:
            r.step("profile", fam, profile_cmds(fam, run_dir), timeout=900.0)
    r.write()
    summary = {"run_dir": str(run_dir), "families": families, "stages": stages,
               "passed": not r.failed and all(x["status"] == "passed" for x in r.records),
               "records": r.records}
    if seal:
        from ..utils.provenance import seal_run

        seal_run(run_dir, command=[PY, "-m", "packmla.bench.kernel_runner"] + sys.argv[1:],
                 extra={"families": families, "stages": stages, "passed": summary["passed"]})
    return summary


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("run_dir", type=Path)
    ap.add_argument("--families", default="decode,store")
    ap.add_argument("--stages", default="build,validate,bench")
    a = ap.parse_args(argv)
    out = run(a.run_dir, a.families.split(","), a.stages.split(","))
    print(json.dumps({k: out[k] for k in ("run_dir", "passed")}))
    return 0 if out["passed"] else 1


if __name__ == "__main__":
    sys.exit(main())

"""Exact scalar Packed evaluation of a policy, mask-method comparison and retention sweep.

    python -m packmla.training.evaluate --cache CACHE --policy POLICY --output out.json [--layers 2,4]
    python -m packmla.training.evaluate --compare-masks   ... --output compare.json [--split all]
    python -m packmla.training.evaluate --retention-sweep ... --output sweep.json

Reference: training/evaluate.py.  Methods at 256 and 192 survivors (MASK_METHODS): magnitude
(TopMag), structured 2:4 / 3:8 over consecutive pre-RoPE coordinates, and the learned scorer; the
sweep covers 64..448 survivors in steps of 64 with magnitude, structured N:8 and learned masks.
Non-256 budgets replay through the dense codec simulation, admitted only after the three 256 masks of
each query reproduce the real codec bit for bit.  Statistics: per issue/layer query means, then
layers and issues equally (mean); pooled query-layer p95 (linear); 10,000 whole-issue bootstrap draws
(seed 42) for 95 % intervals of the mean and of the paired difference to magnitude at the same budget.
Outputs: JSON (complete results) + CSV + Markdown summary (+ PNG curves of a retention sweep),
published only to fresh paths, JSON last.
"""
from __future__ import annotations

import argparse
import csv
import json
from collections import defaultdict
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import parse_layers
from .calibration import Math, reference
from .data.cache import load_cached_layer
from .losses import RETENTION_COUNTS, forward_error, measure, packed_rows, simulated_packed_rows
from .models import StaticScore, read_checkpoint, read_policy, restored_model


@dataclass(frozen=True)
class MaskMethod:
    key: str
    label: str
    retained: int
    group_size: int = 512


MASK_METHODS = (
    MaskMethod("topmag_256", "magnitude (TopMag)", 256),
    MaskMethod("structured_256", "structured 2:4", 256, 4),
    MaskMethod("learned_256", "learned", 256),
    MaskMethod("topmag_192", "magnitude (TopMag)", 192),
    MaskMethod("structured_192", "structured 3:8", 192, 8),
    MaskMethod("learned_192", "learned", 192),
)
SWEEP_METHODS = tuple(
    MaskMethod(f"{fam}_{k}", label, k, 8 if fam == "structured" else 512)
    for k in RETENTION_COUNTS
    for fam, label in (("topmag", "magnitude (TopMag)"), ("structured", "structured N:8"), ("learned", "learned")))
BOOTSTRAP_SAMPLES = 10_000
BOOTSTRAP_SEED = 42


def ranking_mask(scores: torch.Tensor, retained: int, *, group_size: int = 512) -> torch.Tensor:
    """Keep the highest scores globally (group 512) or in every group of `group_size` consecutive
    coordinates; the pruned ones are the smallest per group (torch.topk(largest=False) order on ties)."""
    if (scores.ndim != 2 or scores.shape[-1] != 512 or scores.dtype != torch.float32
            or not bool(torch.isfinite(scores).all()) or retained not in RETENTION_COUNTS
            or group_size not in (4, 8, 512) or retained * group_size % 512):
        raise ValueError("finite FP32 [rows,512] scores and an integral supported mask budget required")
    g = scores.reshape(scores.shape[0], 512 // group_size, group_size)
    mask = torch.ones_like(g, dtype=torch.bool)
    prune = group_size - retained * group_size // 512
    mask.scatter_(-1, g.topk(prune, dim=-1, largest=False).indices, False)
    return mask.reshape_as(scores)


def comparison_masks(raw: torch.Tensor, scores: torch.Tensor, methods=MASK_METHODS) -> dict[str, torch.Tensor]:
    if scores.shape != raw.shape:
        raise ValueError("learned scores must match raw rows")
    return {m.key: ranking_mask(scores if m.key.startswith("learned") else raw.abs(), m.retained,
                                group_size=m.group_size) for m in methods}


def summarize_comparison(records: dict[str, list[dict]], expected: set, methods=MASK_METHODS) -> list[dict]:
    if not expected or set(records) != {m.key for m in methods}:
        raise ValueError("all comparison methods and nonempty expected identities required")
    issues = sorted({rid for rid, _, _ in expected})
    layers = sorted({layer for _, layer, _ in expected})
    draws = np.random.default_rng(BOOTSTRAP_SEED).integers(len(issues), size=(BOOTSTRAP_SAMPLES, len(issues)))
    out, vectors, samples = [], {}, {}
    for m in methods:
        rows = records[m.key]
        keys = [(r["rid"], r["layer"], r["ordinal"]) for r in rows]
        errs = np.asarray([r["error"] for r in rows], dtype=np.float64)
        if len(keys) != len(set(keys)) or set(keys) != expected or not np.isfinite(errs).all() or (errs < 0).any():
            raise ValueError(f"{m.key}: duplicate, missing, mismatched or nonfinite comparison records")
        groups = defaultdict(list)
        for r in rows:
            groups[r["rid"], r["layer"]].append(r["error"])
        means = {k: float(np.mean(v)) for k, v in groups.items()}
        vec = np.asarray([np.mean([means[rid, layer] for layer in layers]) for rid in issues])
        vectors[m.key] = vec
        samples[m.key] = vec[draws].mean(axis=1)
        out.append({
            "method": m.key, "label": m.label, "retained_features": m.retained, "count": len(rows),
            "mean": float(vec.mean()), "p95": float(np.quantile(errs, 0.95, method="linear")),
            "mean_ci95": np.quantile(samples[m.key], [0.025, 0.975]).tolist(),
            "issue_means": dict(zip(issues, vec.tolist())),
            "per_layer": {str(layer): {"mean": float(np.mean([means[rid, layer] for rid in issues])),
                                       "p95": float(np.quantile([r["error"] for r in rows if r["layer"] == layer],
                                                                0.95, method="linear"))} for layer in layers},
            "structured_pattern": (f"{m.retained * m.group_size // 512}:{m.group_size}"
                                   if m.key.startswith("structured") else None)})
    for row in out:
        base = f"topmag_{row['retained_features']}"
        row["paired_vs_magnitude"] = {
            "baseline": base, "mean_difference": float((vectors[row["method"]] - vectors[base]).mean()),
            "mean_difference_ci95": np.quantile(samples[row["method"]] - samples[base], [0.025, 0.975]).tolist()}
    return out


def _fresh(paths: list[Path]) -> None:
    taken = [str(p) for p in paths if p.exists()]
    if taken:
        raise ValueError(f"fresh output paths required (exists: {', '.join(taken)})")


def _write_reports(output: Path, result: dict, created: list[Path]) -> list[str]:
    """CSV, Markdown and (retention sweep) PNG reports, drawn by matplotlib when it is installed and by
    `packmla.utils.png_plot` otherwise; every file is appended to
    `created` as soon as it exists so that a failure can remove the partial report."""
    fields = ("method", "retained_features", "mean", "p95")
    with output.with_suffix(".csv").open("x", newline="") as f:
        created.append(output.with_suffix(".csv"))  # only after the exclusive create succeeded
        w = csv.DictWriter(f, fieldnames=fields)
        w.writeheader()
        w.writerows({k: row[k] for k in fields} for row in result["summary"])
    title = "Attention-error retention sweep" if result.get("retention_sweep") else "Mask-method comparison"
    lines = [f"# {title}", "", f"Split: {result['split']} (reused data, not a fresh held-out test).", "",
             "| Method | Retained | Mean relative output error | p95 | mean 95% CI |", "|---|---:|---:|---:|---|"]
    for row in result["summary"]:
        lo, hi = row["mean_ci95"]
        lines.append(f"| {row['label']} | {row['retained_features']} | {100 * row['mean']:.4f}% | "
                     f"{100 * row['p95']:.4f}% | [{100 * lo:.4f}%, {100 * hi:.4f}%] |")
    cov = result["coverage"]
    lines += ["", f"Coverage: {cov['issues']} issues x {cov['layers']} layers, {cov['query_layer_examples']} "
                  "query-layer examples per method.",
              "The learned scorer was trained at 256 survivors and is reused unchanged at other budgets.", ""]
    with output.with_suffix(".md").open("x") as f:
        created.append(output.with_suffix(".md"))
        f.write("\n".join(lines))
    files = [str(output.with_suffix(".csv")), str(output.with_suffix(".md"))]
    if result.get("retention_sweep"):
        rows = {r["method"]: r for r in result["summary"]}
        try:
            import matplotlib

            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except ImportError:  # the built-in PNG writer: same curves, legend in the report and the PNG's text
            from ..utils.png_plot import line_chart

            result["figures"] = {"renderer": "packmla.utils.png_plot"}
            for metric in ("mean", "p95"):
                path = output.parent / f"{output.stem}-{metric}.png"
                created.append(path)
                info = line_chart(path, list(RETENTION_COUNTS),
                                  {fam: [100 * rows[f"{fam}_{k}"][metric] for k in RETENTION_COUNTS]
                                   for fam in ("topmag", "structured", "learned")},
                                  title=f"{title}: {metric}", xlabel="retained latent coordinates (of 512)",
                                  ylabel=f"{metric} relative output error (%)")
                result["figures"][metric] = info["legend"]
                files.append(str(path))
            return files
        for metric in ("mean", "p95"):
            fig, ax = plt.subplots(figsize=(8, 5))
            for fam in ("topmag", "structured", "learned"):
                ax.plot(RETENTION_COUNTS, [100 * rows[f"{fam}_{k}"][metric] for k in RETENTION_COUNTS], marker="o",
                        label=fam)
            ax.set(xlabel="retained latent coordinates (of 512)", ylabel=f"{metric} relative output error (%)")
            ax.legend()
            path = output.parent / f"{output.stem}-{metric}.png"
            created.append(path)
            fig.savefig(path, dpi=150)
            plt.close(fig)
            files.append(str(path))
    return files


def _states(cache, layer, split):
    roles = ("train", "development") if split == "all" else ("development",)
    states = load_cached_layer(cache, layer)
    return [s for role in roles for s in states[role]]


def compare_masks(cache: Path, policy: Path, output: Path, *, layers: tuple[int, ...], threads: int = 4,
                  retention_sweep: bool = False, split: str = "development") -> dict:
    """Inference-only comparison over the requested layers (CPU)."""
    if split not in ("development", "all"):
        raise ValueError("comparison split must be development or all")
    output = Path(output)
    if output.suffix != ".json":
        raise ValueError("output must be a .json path")
    _fresh([output, output.with_suffix(".csv"), output.with_suffix(".md")]
           + ([output.parent / f"{output.stem}-{m}.png" for m in ("mean", "p95")] if retention_sweep else []))
    torch.set_num_threads(threads)
    math, ref = Math(), reference()
    allowed = tuple(json.loads((Path(cache) / "config.json").read_text())["layers"])
    selected = read_policy(Path(policy), allowed)
    for layer in layers:
        if layer not in selected:
            raise ValueError(f"policy missing requested layer: {layer}")
        read_checkpoint(selected[layer])
    methods = SWEEP_METHODS if retention_sweep else MASK_METHODS
    records = {m.key: [] for m in methods}
    expected = set()
    with torch.no_grad():
        for layer in layers:
            model = restored_model(read_checkpoint(selected[layer])["selected_parameters"], "cpu", 42 + layer).eval()
            for st in _states(cache, layer, split):
                ident = f"{st['rid']}/layer-{layer}/query-{st['ordinal']}"
                expected.add((st["rid"], layer, st["ordinal"]))
                masks = comparison_masks(st["raw"], model(st["raw"], st["eps"]), methods)
                for m in methods:
                    if m.retained == 256:
                        args = (math, ref, st["raw"], masks[m.key], st["weight"], st["eps"], st["freq"])
                        if not torch.equal(packed_rows(*args), simulated_packed_rows(*args)):
                            raise ValueError(f"{ident}/{m.key}: dense codec differs from the 256 codec")
                for m in methods:
                    e = float(forward_error(math, ref, st, model, keep_mask=masks[m.key], retained_features=m.retained))
                    if not np.isfinite(e):
                        raise ValueError(f"{ident}/{m.key}: nonfinite output error")
                    records[m.key].append({"rid": st["rid"], "layer": layer, "ordinal": st["ordinal"], "error": e})
    summary = summarize_comparison(records, expected, methods)
    result = {"schema_version": 1, "status": "complete", "split": split, "retention_sweep": retention_sweep,
              "summary": summary, "records": records,
              "coverage": {"issues": len({r for r, _, _ in expected}), "layers": len(layers),
                           "query_layer_examples": len(expected)},
              "settings": {"cache": str(Path(cache).resolve()), "policy": str(Path(policy).resolve()),
                           "torch": torch.__version__, "threads": threads}}
    # the JSON is the completion marker, written last; any failure removes the partial report
    # (reference: training/evaluate.py report publication, tested by its report-rollback case)
    created: list[Path] = []
    try:
        result["files"] = _write_reports(output, result, created)
        Math.atomic_json(output, result)
    except BaseException:
        for path in created + [output]:
            path.unlink(missing_ok=True)
        raise
    return {"output": str(output), "summary": [{k: r[k] for k in ("method", "mean", "p95")} for r in summary]}


def evaluate(cache: Path, policy: Path, output: Path, *, layers: tuple[int, ...], threads: int = 4) -> dict:
    """Diagnostic development replay of a policy: learned scorer vs TopMag per layer."""
    output = Path(output)
    _fresh([output])
    torch.set_num_threads(threads)
    math, ref = Math(), reference()
    allowed = tuple(json.loads((Path(cache) / "config.json").read_text())["layers"])
    selected = read_policy(Path(policy), allowed)
    per_layer = {}
    for layer in layers:
        model = restored_model(read_checkpoint(selected[layer])["selected_parameters"], "cpu", 42 + layer).eval()
        dev = load_cached_layer(cache, layer)["development"]
        base, _ = measure(math, ref, dev, StaticScore(torch.zeros(512)))
        learned, records = measure(math, ref, dev, model)
        per_layer[str(layer)] = {"topmag": base, "learned": learned, "records": records,
                                 "reduction_percent": 100 * (1 - learned["mean"] / base["mean"])}
    result = {"schema_version": 1, "status": "complete", "split": "development", "layers": list(layers),
              "per_layer": per_layer,
              "mean_topmag": float(np.mean([v["topmag"]["mean"] for v in per_layer.values()])),
              "mean_learned": float(np.mean([v["learned"]["mean"] for v in per_layer.values()]))}
    Math.atomic_json(output, result)
    return {k: result[k] for k in ("mean_topmag", "mean_learned", "layers")}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--cache", type=Path, required=True)
    ap.add_argument("--policy", type=Path, required=True)
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--runner", type=Path, help="accepted for CLI compatibility; packmla's oracle is built in")
    ap.add_argument("--layers", default=None)
    ap.add_argument("--threads", type=int, default=4)
    mode = ap.add_mutually_exclusive_group()
    mode.add_argument("--compare-masks", action="store_true")
    mode.add_argument("--retention-sweep", action="store_true")
    ap.add_argument("--split", choices=("development", "all"), default="development")
    a = ap.parse_args(argv)
    allowed = tuple(json.loads((a.cache / "config.json").read_text())["layers"])
    layers = parse_layers(a.layers, allowed) if a.layers else allowed
    if a.compare_masks or a.retention_sweep:
        return compare_masks(a.cache, a.policy, a.output, layers=layers, threads=a.threads,
                             retention_sweep=a.retention_sweep, split=a.split)
    return evaluate(a.cache, a.policy, a.output, layers=layers, threads=a.threads)


if __name__ == "__main__":
    print(json.dumps(main(), indent=2))

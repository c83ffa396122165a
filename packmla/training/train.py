"""Fit rank-64 conditional scorers per C4 layer and publish a policy.

    python -m packmla.training.train --cache CACHE --policy POLICY --output OUT --recipe continuation \
        [--layers 2,4] [--device cpu|cuda] [--threads 4]
    python -m packmla.training.train --init-policy OUT --cache CACHE   # fresh rank-16 starting policy

Reference: training/train.py (fit :91-372, run :374-510, CLI :512-534).  Same objective and
selection rule:

* per epoch: geometric temperature schedule T_start -> T_end; Adam with per-group learning rates
  (theta 3e-3, encoders 1e-3, decoders 3e-3, times the recipe's scale); per-query loss
  e + 2 relu(e - e_TopMag), weighted 1 / (issues * queries of its issue); L2 penalty 1e-3 on theta and
  the decoders; gradient clip 1; theta clamped to +-bound;
* a candidate is selected only if its development mean beats the best so far and neither its mean nor
  its p95 is worse than TopMag (`validation_acceptable`); otherwise the warm scorer is kept;
* outputs never overwrite: a fresh output directory, per-layer checkpoint JSON, and `policy.json`
  published last (atomically) as the completion marker, with untouched layers inherited.
"""
from __future__ import annotations

import argparse
import copy
import json
import os
from collections import Counter
from pathlib import Path

import numpy as np
import torch

from . import parse_layers
from .calibration import Math, reference
from .data.batches import StateBatches
from .data.cache import load_cached_layer
from .losses import codec_residual_anchor, forward_error, measure, select_objective, validation_acceptable
from .models import (ExpandedConditionalScore, StaticScore, extend_parameters, initial_rank16_parameters,
                     read_checkpoint, read_policy)

RECIPES = json.loads((Path(__file__).parent / "recipes.json").read_text())


def parameter_penalty(model: ExpandedConditionalScore) -> torch.Tensor:
    return 0.001 * sum(p.square().mean() for p in (model.theta, model.decoder, model.decoder_even,
                                                    model.extra_decoder, model.extra_decoder_even))


def parameter_groups(model: ExpandedConditionalScore, scale: float) -> list[dict]:
    return [{"params": [model.theta], "lr": 0.003 * scale},
            {"params": [model.encoder, model.extra_encoder], "lr": 0.001 * scale},
            {"params": [model.decoder, model.decoder_even, model.extra_decoder, model.extra_decoder_even],
             "lr": 0.003 * scale}]


def _load_parameters(model, parameters: dict, device, theta0, bound) -> None:
    """Warm-start `model` from checkpoint parameters whose theta is the declared initial theta."""
    layout = model.state_dict()
    missing, extra = sorted(set(layout) - set(parameters)), sorted(set(parameters) - set(layout))
    if missing or extra:
        raise ValueError(f"warm start: missing parameters {missing}, unexpected parameters {extra}")
    restored = {}
    for name, ref in layout.items():
        t = torch.as_tensor(parameters[name], device=device, dtype=ref.dtype)
        if t.shape != ref.shape or not bool(torch.isfinite(t).all()):
            raise ValueError(f"warm start: {name!r} must be finite with shape {tuple(ref.shape)}")
        restored[name] = t
    if float(restored["theta"].abs().max()) > bound + 1e-7:
        raise ValueError(f"warm start: theta leaves the trust region |theta| <= {bound}")
    if not torch.equal(restored["theta"], theta0):
        raise ValueError("warm start: the checkpoint's theta is not the initial theta given to fit()")
    model.load_state_dict(restored)


def _check_fit_arguments(train, development, mode, epochs, bound, train_batch_size, learning_rate_scale,
                         temperature_start, temperature_end) -> None:
    """Reject a fit whose settings leave the ranges the recipes use, or whose data splits overlap."""
    problems = []
    if mode != "conditional_expanded":
        problems.append(f"mode {mode!r} (only conditional_expanded is trained)")
    if not 1 <= epochs <= 100:
        problems.append(f"epochs {epochs!r} outside 1..100")
    if not 0 < bound <= 1:
        problems.append(f"trust-region bound {bound!r} outside (0, 1]")
    if not isinstance(train_batch_size, int) or not 1 <= train_batch_size <= 16:
        problems.append(f"train_batch_size {train_batch_size!r} outside 1..16")
    if not 0 < learning_rate_scale <= 1:
        problems.append(f"learning_rate_scale {learning_rate_scale!r} outside (0, 1]")
    if not 0 < temperature_end <= temperature_start <= 0.15:
        problems.append(f"temperatures {temperature_start!r} -> {temperature_end!r} not a descending schedule "
                        "inside (0, 0.15]")
    if not train or not development:
        problems.append("an empty training or development split")
    elif any(st.get("role") != "train" for st in train):
        problems.append("training states not marked role='train'")
    elif {st["rid"] for st in train} & {st["rid"] for st in development}:
        problems.append("issues shared by the training and development splits")
    if problems:
        raise ValueError("fit: " + "; ".join(problems))


def fit(math, ref, train: list[dict], development: list[dict], initial_theta: torch.Tensor, *,
        mode: str = "conditional_expanded", epochs: int = 40, bound: float = 0.5, seed: int = 42,
        checkpoint=None, initial_parameters: dict | None = None, learning_rate_scale: float = 1.0,
        temperature_start: float = 0.03, temperature_end: float = 0.015, train_batch_size: int = 1,
        gradient_mode: str = "straight_through", device=None, scratch_root: Path | None = None) -> dict:
    _check_fit_arguments(train, development, mode, epochs, bound, train_batch_size, learning_rate_scale,
                         temperature_start, temperature_end)
    device = torch.device(device) if device is not None else train[0]["raw"].device
    theta0 = initial_theta.detach().to(device)
    if theta0.shape != (512,) or not bool(torch.isfinite(theta0).all()) or float(theta0.abs().max()) > bound + 1e-7:
        raise ValueError(f"fit: initial theta must be 512 finite values with |theta| <= {bound}")
    model = ExpandedConditionalScore(theta0, seed=seed).to(device)
    if initial_parameters is not None:
        _load_parameters(model, initial_parameters, device, theta0, bound)
    params = tuple(p for p in model.parameters() if p.requires_grad)
    warm = StaticScore(theta0) if initial_parameters is None else copy.deepcopy(model)
    baseline = StaticScore(torch.zeros_like(theta0))
    base_metrics, _ = measure(math, ref, development, baseline)
    warm_metrics, _ = measure(math, ref, development, warm)
    if initial_parameters is not None and not validation_acceptable(warm_metrics, base_metrics):
        raise ValueError("fit: the warm start is worse than TopMag on the development split (mean or p95)")
    with StateBatches(train, device, train_batch_size, scratch_root) as batches:
        obj = select_objective(math, ref, model, gradient_mode)
        if obj.anchored:
            batches.prepare_anchors(lambda st: codec_residual_anchor(math, ref, st, warm))
        # gradient preflight: the straight-through surrogate must equal the exact error in value
        t_pre = 0.03 if gradient_mode == "straight_through" else temperature_start
        with batches.stage([0]) as b:
            exact = forward_error(math, ref, b.states[0], model)
            sur = obj.scalar(b.states, t_pre, b.anchors)
            if gradient_mode == "straight_through":
                torch.testing.assert_close(sur.detach(), exact.detach(), atol=0, rtol=0)
            if not all(bool(torch.isfinite(g).all()) for g in torch.autograd.grad(sur, params)):
                raise ValueError("fit: the first training state's gradient has non-finite entries")
        batch_check = None
        if train_batch_size > 1:
            with batches.stage(range(min(train_batch_size, len(train)))) as b:
                batch_check = obj.preflight(b.states, temperature_start, b.anchors)
        opt = torch.optim.Adam(parameter_groups(model, learning_rate_scale))
        best, best_metrics = None, warm_metrics
        init_metrics = warm_metrics if initial_parameters is not None else measure(math, ref, development, model)[0]
        if validation_acceptable(init_metrics, base_metrics) and init_metrics["mean"] < best_metrics["mean"]:
            best, best_metrics = copy.deepcopy(model.state_dict()), init_metrics
        with torch.no_grad():
            train_base = []
            for i in range(len(train)):
                with batches.stage([i], with_anchors=False) as b:
                    train_base.append(float(forward_error(math, ref, b.states[0], baseline)))
        counts = Counter(s["rid"] for s in train)
        weight_of = [1.0 / (len(counts) * counts[s["rid"]]) for s in train]
        rng = np.random.default_rng(seed)
        history = []
        snapshot = None
        for epoch in range(epochs):
            T = temperature_start * (temperature_end / temperature_start) ** (epoch / max(epochs - 1, 1))
            opt.zero_grad()
            losses = []
            order = rng.permutation(len(train))
            for start in range(0, len(train), train_batch_size):
                idx = order[start:start + train_batch_size]
                with batches.stage(idx) as b:
                    if train_batch_size == 1:
                        e = obj.scalar(b.states, T, b.anchors)
                        i = int(idx[0])
                        loss = (e + 2 * torch.relu(e - train_base[i])) * weight_of[i]
                    else:
                        e = obj.batch(b.states, T, b.anchors)
                        base = e.new_tensor([train_base[i] for i in idx])
                        w = e.new_tensor([weight_of[i] for i in idx])
                        loss = ((e + 2 * torch.relu(e - base)) * w).sum()
                    loss.backward()
                    losses.append(float(loss.detach()))
            total = float(sum(losses))
            parameter_penalty(model).backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0, error_if_nonfinite=True)
            opt.step()
            with torch.no_grad():
                model.theta.clamp_(-bound, bound)
            sat = float((model.theta.abs() >= bound - 1e-6).float().mean())
            metrics, _ = measure(math, ref, development, model)
            accepted = validation_acceptable(metrics, base_metrics) and metrics["mean"] < best_metrics["mean"]
            if accepted:
                best, best_metrics = copy.deepcopy(model.state_dict()), metrics
            history.append({"epoch": epoch + 1, "temperature": T, "train_objective": total, "development": metrics,
                            "checkpoint_selected": accepted, "bound_fraction": sat})
            selected_state = (None if initial_parameters is None else warm.state_dict()) if best is None else best
            snapshot = {"mode": mode, "gradient_mode": gradient_mode,
                        "selected_parameters": None if selected_state is None else
                        {k: v.tolist() for k, v in selected_state.items()},
                        "current_parameters": {k: v.detach().tolist() for k, v in model.state_dict().items()},
                        "warm_theta": theta0.tolist(), "warm_mode": mode if initial_parameters is not None else "static",
                        "development_selected": best_metrics, "history": history}
            if checkpoint is not None:
                checkpoint(snapshot)
            print(f"{mode} epoch {epoch + 1}/{epochs}: {metrics['mean']:.8f}, selected={accepted}", flush=True)
        if best is None:
            selected_model = warm
        else:
            model.load_state_dict(best)
            selected_model = model
        sel_metrics, records = measure(math, ref, development, selected_model)
        result = {**snapshot, "development_baseline": base_metrics, "development_warm": warm_metrics,
                  "batch_preflight": batch_check, "train_batch_size": train_batch_size,
                  "development_selected": sel_metrics, "selected_records": records, "fallback_to_warm": best is None,
                  "reduction_percent": 100 * (1 - sel_metrics["mean"] / base_metrics["mean"])}
        if obj.anchored:
            result.update(codec_anchor_policy="frozen_warm", codec_anchor_queries=len(train),
                          codec_anchor_bytes=batches.anchor_bytes)
        if result["selected_parameters"] is None:  # no warm model and nothing accepted: keep the static warm
            result["selected_parameters"] = {k: v.tolist() for k, v in
                                              ExpandedConditionalScore(theta0.cpu(), seed=seed).state_dict().items()}
        return result


def _exact_fp32_matmuls() -> None:
    """Candidates are ranked by attention errors that differ in the fourth digit: fp32 products stay fp32
    (no TF32 on either matmul path)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")


def _cache_layers(cache: Path) -> tuple[int, ...]:
    return tuple(json.loads((Path(cache) / "config.json").read_text())["layers"])


def init_policy(cache: Path, output: Path, seed: int = 42) -> dict:
    """Write rank-16 starting checkpoints (theta 0, zero decoders) for every cached layer + a policy."""
    output = Path(output)
    if output.exists():
        raise ValueError(f"{output} exists: init_policy writes into a new directory only")
    output.mkdir(parents=True)
    entries = []
    for layer in _cache_layers(cache):
        path = output / f"init-layer-{layer:02d}.json"
        Math.atomic_json(path, {"layer": layer, "selected_parameters": initial_rank16_parameters(seed + layer),
                                "mode": "rank16_init"})
        entries.append({"layer": layer, "path": path.name})
    Math.atomic_json(output / "policy.json", {"selected": entries, "trained_layers": []})
    return {"policy": str(output / "policy.json"), "layers": [e["layer"] for e in entries]}


def run(cache: Path, policy: Path, output: Path, *, recipe: str, layers: tuple[int, ...], device: str = "cpu",
        threads: int = 4, epochs: int | None = None) -> dict:
    if recipe not in RECIPES:
        raise ValueError(f"recipe {recipe!r} is not one of {sorted(RECIPES)}")
    if threads < 1 or device not in ("cpu", "cuda"):
        raise ValueError(f"threads {threads!r} / device {device!r}: need threads >= 1 and device cpu or cuda")
    output = Path(output)
    if output.exists():
        raise ValueError(f"{output} exists: a training run writes into a new directory only")
    if device == "cuda" and not torch.cuda.is_available():
        raise ValueError("device cuda was asked for but no GPU is visible (training does not fall back to the CPU)")
    math, ref = Math(), reference()
    torch.set_num_threads(threads)
    _exact_fp32_matmuls()
    allowed = _cache_layers(cache)
    selected = read_policy(Path(policy), allowed)
    missing = sorted(set(layers) - selected.keys())
    if missing:
        raise ValueError(f"the policy has no checkpoint for layers {missing}")
    records = {layer: read_checkpoint(e) for layer, e in selected.items() if layer in layers}
    settings = dict(RECIPES[recipe])
    if epochs is not None:
        settings["epochs"] = epochs
    output.mkdir(parents=True)
    Math.atomic_json(output / "config.json", {"recipe": recipe, "settings": settings, "layers": list(layers),
                                              "cache": str(Path(cache).resolve()), "policy": str(Path(policy).resolve()),
                                              "torch": torch.__version__, "device": device, "threads": threads})
    done = []
    for layer in layers:
        states = load_cached_layer(cache, layer)
        params = records[layer]["selected_parameters"]
        if recipe == "rank64":
            params = extend_parameters(params, 42 + layer)
        result = fit(math, ref, states["train"], states["development"], torch.tensor(params["theta"], device=device),
                     seed=42 + layer, initial_parameters=params, device=device, scratch_root=output,
                     checkpoint=lambda part, layer=layer: Math.atomic_json(output / f"partial-layer-{layer:02d}.json",
                                                                           part),
                     **settings)
        result["layer"] = layer
        path = output / f"selected-layer-{layer:02d}.json"
        Math.atomic_json(path, result)
        selected[layer] = {"layer": layer, "path": str(path.resolve())}
        done.append(layer)
        Math.atomic_json(output / "progress.json", {"layers": done, "complete": False})
    published = []
    for layer, e in sorted(selected.items()):
        read_checkpoint(e)
        published.append({**e, "path": Path(e["path"]).name} if layer in layers else e)
    # the policy is the completion marker: staged under a temporary name, hard-linked into place and
    # checked to be the staged file; any failure (interrupts included) leaves no policy.json behind
    # (reference: training/train.py:448-509)
    tmp = output / ".policy.json.tmp"
    final = output / "policy.json"
    Math.atomic_json(tmp, {"selected": published, "trained_layers": list(layers)})
    linked = False
    try:
        os.link(tmp, final)
        linked = True
        if os.stat(tmp).st_ino != os.stat(final).st_ino:
            raise RuntimeError("published policy is not the staged file")
    except BaseException:
        if linked:
            final.unlink(missing_ok=True)
        raise
    finally:
        try:
            tmp.unlink(missing_ok=True)
        except OSError:  # a staging name left behind does not invalidate the published policy
            pass
    Math.atomic_json(output / "progress.json", {"layers": done, "complete": True})
    return {"layers": done, "output": str(output), "policy": str(output / "policy.json")}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--cache", type=Path, required=True)
    ap.add_argument("--policy", type=Path)
    ap.add_argument("--output", type=Path)
    ap.add_argument("--init-policy", type=Path, help="write a fresh rank-16 starting policy here and exit")
    ap.add_argument("--runner", type=Path, help="accepted for CLI compatibility; packmla's oracle is built in")
    ap.add_argument("--recipe", choices=tuple(RECIPES))
    ap.add_argument("--layers", default=None)
    ap.add_argument("--device", choices=("cpu", "cuda"), default="cpu")
    ap.add_argument("--threads", type=int, default=4)
    ap.add_argument("--epochs", type=int, default=None, help="override the recipe's epoch count")
    a = ap.parse_args(argv)
    if a.init_policy is not None:
        return init_policy(a.cache, a.init_policy)
    if a.policy is None or a.output is None or a.recipe is None:
        ap.error("--policy, --output and --recipe are required for training")
    allowed = _cache_layers(a.cache)
    layers = parse_layers(a.layers, allowed) if a.layers else allowed
    return run(a.cache, a.policy, a.output, recipe=a.recipe, layers=layers, device=a.device, threads=a.threads,
               epochs=a.epochs)


if __name__ == "__main__":
    print(json.dumps(main(), indent=2))

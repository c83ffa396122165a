"""Exact Packed replay losses and the training relaxations of the hard Top-256 mask.

Error of one captured decode query (training/losses.py:148-213, reference semantics):

    rows   = Packed rows of the selected C4 records under the scorer's mask (exact codec: masked
             RMSNorm, BF16, UE8M0/E4M3, RoPE at read time), concatenated after the Native SWA rows
    output = attention(q, rows, sink) with inverse output RoPE, BF16-rounded
    error  = |output - target| / |target|   (target: the same query over Native records)

The hard mask has no gradient.  Three training objectives differentiate a surrogate instead:
  straight_through: forward value = exact error; backward through a continuous path in which the
                    mask is replaced by BudgetGate (a sigmoid gate whose threshold keeps sum = 256);
  relaxed:          forward and backward both on the continuous gated path (no codec rounding);
  anchored:         the relaxed path plus fixed codec residuals measured at the warm scorer's mask.
The exact scalar replay (`forward_error` without temperature) decides between candidates.
Every objective has a scalar and an independent batched implementation; `preflight` checks that both
agree in value and gradient before a fit uses the batched one.
"""
from __future__ import annotations

from collections import defaultdict
from typing import Callable, NamedTuple

import numpy as np
import torch

RETENTION_COUNTS = tuple(range(64, 449, 64))
KEEP = 256


class BudgetGate(torch.autograd.Function):
    """g = sigmoid((s - t) / T) with the threshold t solved (bisection, 48 halvings) so sum(g) = 256.

    Backward is the Jacobian of the smooth gate including dt/ds: with w = g (1 - g),
    dL/ds = w (dL/dg - sum(w dL/dg) / sum(w)) / T, which is invariant to a common shift of the scores.
    """

    @staticmethod
    def forward(ctx, scores: torch.Tensor, temperature: float):
        if temperature <= 0 or scores.shape[-1] != 512:
            raise ValueError("positive temperature and 512 scores required")
        lo = scores.amin(-1, keepdim=True) - 40 * temperature
        hi = scores.amax(-1, keepdim=True) + 40 * temperature
        for _ in range(48):
            mid = (lo + hi) / 2
            over = torch.sigmoid((scores - mid) / temperature).sum(-1, keepdim=True) > KEEP
            lo = torch.where(over, mid, lo)
            hi = torch.where(over, hi, mid)
        gate = torch.sigmoid((scores - (lo + hi) / 2) / temperature)
        ctx.save_for_backward(gate)
        ctx.temperature = temperature
        return gate

    @staticmethod
    def backward(ctx, grad):
        (gate,) = ctx.saved_tensors
        w = gate * (1 - gate)
        centre = (w * grad).sum(-1, keepdim=True) / w.sum(-1, keepdim=True).clamp_min(1e-30)
        return w * (grad - centre) / ctx.temperature, None


# ----------------------------------------------------------------------------- codec views
def _check_mask(raw: torch.Tensor, mask: torch.Tensor, kept: int) -> None:
    if kept not in RETENTION_COUNTS:
        raise ValueError("retained features must be 64 through 448 in multiples of 64")
    if (mask.dtype != torch.bool or mask.shape != raw.shape or raw.ndim != 2 or raw.shape[-1] != 512
            or not bool((mask.sum(-1) == kept).all())):
        raise ValueError(f"bool mask matching raw rows with exactly {kept} survivors required")


def simulated_packed_rows(math, ref, raw, mask, weight, eps, freqs, *, retained_features: int = KEEP):
    """Dense simulation of any budget with the 256 codec's rounding (offline only, not a record)."""
    from ..formats import codec

    _check_mask(raw, mask, retained_features)
    return codec.simulated_packed_rows(raw.float(), mask, weight, eps, freqs)


def packed_rows(math, ref, raw, mask, weight, eps, freqs, *, retained_features: int = KEEP):
    """Rows a Direct reader sees: the real 256-value codec, or the dense simulation for other budgets."""
    _check_mask(raw, mask, retained_features)
    if retained_features != KEEP:
        return simulated_packed_rows(math, ref, raw, mask, weight, eps, freqs, retained_features=retained_features)
    values, bitmap, scales = ref.pack_rows_ref(raw, mask, weight, eps)
    return math.rotate(ref.unpack_rows_ref(values, bitmap, scales).float(), freqs).to(torch.bfloat16).float()


def rounded_output(math, value, freqs):
    """BF16 output, inverse RoPE of the tail at the query position, BF16 again."""
    return math.rotate(value.to(torch.bfloat16).float(), freqs, True).to(torch.bfloat16).float()


def _continuous_rows(math, raw, gate, weight, eps, freqs):
    x = raw * gate
    return math.rotate(x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * weight, freqs)


def _hard_mask(model, ref, raw, eps, scores, kept: int = KEEP) -> torch.Tensor:
    if kept == KEEP and hasattr(model, "hard_mask"):
        return model.hard_mask(ref, raw, eps)
    mask = torch.ones_like(scores, dtype=torch.bool)
    mask.scatter_(-1, scores.detach().topk(512 - kept, dim=-1, largest=False).indices, False)
    return mask


def _relative(output, target, denom):
    sq = (output - target).square().sum(dim=(-2, -1)).to(torch.float64)
    return (sq / denom).clamp_min(1e-30).sqrt()


def _training_only(state: dict, what: str) -> None:
    """Gradients, the continuous relaxation and codec anchors exist only for states of the training split."""
    if state.get("role") != "train":
        raise ValueError(f"{what}: state of role {state.get('role')!r}; only the training split may use it")


def _relaxation_temperature(t: float) -> None:
    if not 0 < t <= 0.15:
        raise ValueError(f"relaxation temperature {t!r} outside (0, 0.15]")


# ----------------------------------------------------------------------------- scalar (the deciding replay)
def forward_error(math, ref, state: dict, model, temperature: float | None = None, *,
                  retained_features: int = KEEP, keep_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Exact Packed attention error of one state; with `temperature`, straight-through gradients."""
    if temperature is not None and (retained_features != KEEP or keep_mask is not None):
        raise ValueError(f"gradients run at the serving budget of {KEEP} with the scorer's own mask; "
                         "explicit masks and other budgets are for evaluation")
    if retained_features not in RETENTION_COUNTS:
        raise ValueError(f"retained_features {retained_features!r} not in {RETENTION_COUNTS}")
    scores = None
    if keep_mask is not None:
        mask = keep_mask
    else:
        scores = model(state["raw"], state["eps"])
        mask = _hard_mask(model, ref, state["raw"], state["eps"], scores, retained_features)
    with torch.no_grad():
        exact = packed_rows(math, ref, state["raw"], mask, state["weight"], state["eps"], state["freq"],
                            retained_features=retained_features)
    rows = exact
    if temperature is not None:
        _training_only(state, "straight-through gradient")
        soft = BudgetGate.apply(scores, temperature)
        gate = mask.float() + (soft - soft.detach())
        cont = _continuous_rows(math, state["raw"], gate, state["weight"], state["eps"], state["freq"])
        rows = exact + (cont - cont.detach())
    out = math.attention(state["q"], torch.cat((state["swa"], rows)), state["sink"], state["scale"])[0]
    exact_out = rounded_output(math, out.detach(), state["query_freq"])
    if temperature is None:
        out = exact_out
    else:
        cont = math.rotate(out, state["query_freq"], True)
        out = exact_out + (cont - cont.detach())
    return _relative(out[None], state["target"][None], state["reference_squared_norm"])[0]


def relaxed_forward_error(math, state: dict, model, temperature: float, anchor: dict | None = None):
    """Continuous gated path (training only); with `anchor`, plus the fixed codec residuals."""
    _training_only(state, "continuous relaxation")
    _relaxation_temperature(temperature)
    if anchor is not None:
        validate_codec_anchor(state, anchor)
    gate = BudgetGate.apply(model(state["raw"], state["eps"]), temperature)
    rows = _continuous_rows(math, state["raw"], gate, state["weight"], state["eps"], state["freq"])
    if anchor is not None:
        rows = rows + anchor["rows"]
    out = math.attention(state["q"], torch.cat((state["swa"], rows)), state["sink"], state["scale"])[0]
    out = math.rotate(out, state["query_freq"], True)
    if anchor is not None:
        out = out + anchor["output"]
    return _relative(out[None], state["target"][None], state["reference_squared_norm"])[0]


def anchored_relaxed_forward_error(math, state, model, temperature, anchor):
    return relaxed_forward_error(math, state, model, temperature, anchor)


def codec_residual_anchor(math, ref, state: dict, model) -> dict:
    """Codec residuals at `model`'s hard mask, held fixed while training (not a serving input)."""
    _training_only(state, "codec anchor")
    with torch.no_grad():
        scores = model(state["raw"], state["eps"])
        mask = torch.ones_like(scores, dtype=torch.bool)
        mask.scatter_(-1, scores.topk(KEEP, dim=-1, largest=False).indices, False)
        cont = _continuous_rows(math, state["raw"], mask.float(), state["weight"], state["eps"], state["freq"])
        packed = packed_rows(math, ref, state["raw"], mask, state["weight"], state["eps"], state["freq"])
        out = math.attention(state["q"], torch.cat((state["swa"], packed)), state["sink"], state["scale"])[0]
        return {"state": state, "rows": (packed - cont).detach(),
                "output": (rounded_output(math, out, state["query_freq"])
                           - math.rotate(out, state["query_freq"], True)).detach()}


def validate_codec_anchor(state: dict, anchor: dict) -> None:
    _training_only(state, "codec anchor")
    if anchor.get("state") is not state:
        raise ValueError("codec anchor was built for another state object")
    for key, like in (("rows", state["raw"]), ("output", state["target"])):
        v = anchor[key]
        fits = v.shape == like.shape and v.device == like.device and v.dtype == like.dtype
        if not fits or v.requires_grad or not bool(torch.isfinite(v).all()):
            raise ValueError(f"codec anchor {key!r} must be a finite constant shaped like the state's {key}")


# ----------------------------------------------------------------------------- batched
_STACK = ("raw", "weight", "freq", "q", "swa", "sink", "target", "query_freq")


def stack_states(states: list[dict], anchors: list[dict] | None = None) -> dict:
    if not states:
        raise ValueError("stack_states: empty batch")
    first = states[0]
    for i, s in enumerate(states):
        if (s["eps"], s["scale"]) != (first["eps"], first["scale"]):
            raise ValueError(f"stack_states: state {i} is from another layer (epsilon or softmax scale differs)")
        odd = [k for k in _STACK if s[k].shape != first[k].shape]
        if odd:
            raise ValueError(f"stack_states: state {i} differs in shape for {odd}")
    batch = {k: torch.stack([s[k] for s in states]) for k in _STACK}
    batch.update(eps=first["eps"], scale=first["scale"], roles=[s["role"] for s in states],
                 reference_squared_norm=torch.tensor([s["reference_squared_norm"] for s in states],
                                                     dtype=torch.float64, device=first["raw"].device))
    if anchors is not None:
        if len(anchors) != len(states):
            raise ValueError(f"stack_states: {len(anchors)} codec anchors for {len(states)} states")
        for s, a in zip(states, anchors):
            validate_codec_anchor(s, a)
        batch["codec_rows"] = torch.stack([a["rows"] for a in anchors])
        batch["codec_output"] = torch.stack([a["output"] for a in anchors])
    return batch


def _batched_attention(batch, rows):
    kv = torch.cat((batch["swa"], rows), dim=1)
    logits = torch.bmm(batch["q"], kv.transpose(1, 2)) * batch["scale"]
    p = torch.softmax(torch.cat((logits, batch["sink"][..., None]), -1), -1)[..., :-1]
    return torch.bmm(p, kv)


def forward_errors(math, ref, batch: dict, model, temperature: float | None = None) -> torch.Tensor:
    """Batched counterpart of `forward_error` (256 survivors, model masks)."""
    n, rows_per, width = batch["raw"].shape
    raw = batch["raw"].reshape(-1, width)
    freqs = batch["freq"].reshape(-1, batch["freq"].shape[-1])
    weight = batch["weight"][:, None, :].expand(n, rows_per, width).reshape(-1, width)
    scores = model(raw, batch["eps"])
    mask = _hard_mask(model, ref, raw, batch["eps"], scores)
    with torch.no_grad():
        exact = torch.cat([packed_rows(math, ref, raw[i * rows_per:(i + 1) * rows_per],
                                       mask[i * rows_per:(i + 1) * rows_per], batch["weight"][i], batch["eps"],
                                       freqs[i * rows_per:(i + 1) * rows_per]) for i in range(n)])
    rows = exact
    if temperature is not None:
        for role in batch["roles"]:
            _training_only({"role": role}, "straight-through gradient")
        soft = BudgetGate.apply(scores, temperature)
        gate = mask.float() + (soft - soft.detach())
        cont = _continuous_rows(math, raw, gate, weight, batch["eps"], freqs)
        rows = exact + (cont - cont.detach())
    out = _batched_attention(batch, rows.reshape(n, rows_per, width))
    qf = batch["query_freq"][:, None, :]
    exact_out = rounded_output(math, out.detach(), qf)
    if temperature is None:
        out = exact_out
    else:
        cont = math.rotate(out, qf, True)
        out = exact_out + (cont - cont.detach())
    return _relative(out, batch["target"], batch["reference_squared_norm"])


def relaxed_forward_errors(math, batch: dict, model, temperature: float, *, anchored: bool = False):
    for role in batch["roles"]:
        _training_only({"role": role}, "continuous relaxation")
    _relaxation_temperature(temperature)
    n, rows_per, width = batch["raw"].shape
    raw = batch["raw"].reshape(-1, width)
    gate = BudgetGate.apply(model(raw, batch["eps"]), temperature)
    weight = batch["weight"][:, None, :].expand(n, rows_per, width).reshape(-1, width)
    rows = _continuous_rows(math, raw, gate, weight, batch["eps"], batch["freq"].reshape(-1, batch["freq"].shape[-1]))
    if anchored:
        rows = rows + batch["codec_rows"].reshape(-1, width)
    out = math.rotate(_batched_attention(batch, rows.reshape(n, rows_per, width)), batch["query_freq"][:, None, :],
                      True)
    if anchored:
        out = out + batch["codec_output"]
    return _relative(out, batch["target"], batch["reference_squared_norm"])


# ----------------------------------------------------------------------------- checks and metrics
def _compare(vector, scalar, vgrad, sgrad, what: str) -> dict:
    torch.testing.assert_close(vector.detach(), scalar.detach(), atol=2e-6, rtol=2e-5)
    for a, b in zip(vgrad, sgrad):
        if not bool(torch.isfinite(a).all()):
            raise ValueError(f"{what} preflight: the batched gradient has non-finite entries")
        torch.testing.assert_close(a, b, atol=2e-5, rtol=2e-4)
    return {"forward_max_abs": float((vector - scalar).detach().abs().max()),
            "gradient_max_abs": max(float((a - b).abs().max()) for a, b in zip(vgrad, sgrad)),
            "selection": "scalar exact Packed development replay"}


def preflight(math, ref, states: list[dict], model, temperature: float) -> dict:
    """Scalar and batched straight-through paths agree in value and gradient."""
    params = tuple(p for p in model.parameters() if p.requires_grad)
    scalar = torch.stack([forward_error(math, ref, s, model, temperature) for s in states])
    vector = forward_errors(math, ref, stack_states(states), model, temperature)
    sg = torch.autograd.grad(scalar.sum(), params)
    vg = torch.autograd.grad(vector.sum(), params)
    return {"states": len(states), **_compare(vector, scalar, vg, sg, "straight-through")}


def relaxed_preflight(math, states: list[dict], model, temperature: float, anchors=None) -> dict:
    params = tuple(p for p in model.parameters() if p.requires_grad)
    scalar = torch.stack([relaxed_forward_error(math, s, model, temperature, None if anchors is None else a)
                          for s, a in zip(states, anchors or [None] * len(states))])
    vector = relaxed_forward_errors(math, stack_states(states, anchors), model, temperature,
                                    anchored=anchors is not None)
    sg = torch.autograd.grad(scalar.sum(), params)
    vg = torch.autograd.grad(vector.sum(), params)
    return {"states": len(states), **_compare(vector, scalar, vg, sg, "relaxed")}


def aggregate(records: list[dict]) -> dict:
    """Issue-weighted mean (queries within an issue first), pooled p95, per-issue means."""
    groups: dict[str, list[float]] = defaultdict(list)
    for r in records:
        groups[r["rid"]].append(r["error"])
    return {"normalized_mse": float(np.mean([np.mean(np.square(v)) for v in groups.values()])),
            "mean": float(np.mean([np.mean(v) for v in groups.values()])),
            "p95": float(np.quantile([r["error"] for r in records], 0.95)),
            "issue_means": {k: float(np.mean(v)) for k, v in sorted(groups.items())}}


def validation_acceptable(metrics: dict, baseline: dict) -> bool:
    """A candidate may not be worse than TopMag in mean or p95."""
    return metrics["mean"] <= baseline["mean"] and metrics["p95"] <= baseline["p95"]


def measure(math, ref, states: list[dict], model) -> tuple[dict, list[dict]]:
    if not states:
        raise ValueError("measure: no states to measure")
    dev = model.theta.device
    errs = []
    with torch.no_grad():
        for s in states:
            st = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in s.items()}
            errs.append(forward_error(math, ref, st, model))
    values = torch.stack(errs).cpu().tolist()
    records = [{"rid": s["rid"], "ordinal": s["ordinal"], "error": e} for s, e in zip(states, values)]
    return aggregate(records), records


class Objective(NamedTuple):
    scalar: Callable
    batch: Callable
    preflight: Callable
    anchored: bool


def select_objective(math, ref, model, gradient_mode: str) -> Objective:
    """Scalar / batched / preflight callables of one gradient mode (anchors are passed per batch)."""
    if gradient_mode == "straight_through":
        return Objective(lambda st, T, an=None: forward_error(math, ref, st[0], model, T),
                         lambda st, T, an=None: forward_errors(math, ref, stack_states(st), model, T),
                         lambda st, T, an=None: preflight(math, ref, st, model, T), False)
    if gradient_mode == "relaxed":
        return Objective(lambda st, T, an=None: relaxed_forward_error(math, st[0], model, T),
                         lambda st, T, an=None: relaxed_forward_errors(math, stack_states(st), model, T),
                         lambda st, T, an=None: relaxed_preflight(math, st, model, T), False)
    if gradient_mode == "anchored":
        return Objective(lambda st, T, an=None: relaxed_forward_error(math, st[0], model, T, an[0]),
                         lambda st, T, an=None: relaxed_forward_errors(math, stack_states(st, an), model, T,
                                                                       anchored=True),
                         lambda st, T, an=None: relaxed_preflight(math, st, model, T, an), True)
    raise ValueError(f"gradient mode {gradient_mode!r}: use straight_through, relaxed or anchored")

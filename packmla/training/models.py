"""Sensitivity scorers that choose which 256 of 512 latent coordinates a Packed record keeps.

A scorer maps raw FP32 compressor rows [..., 512] (and the RMSNorm epsilon) to per-coordinate
scores; the Packed mask keeps the 256 highest.  The checkpoint parameter names and the arithmetic are
the reference's (training/models.py:81-214), because policies and checkpoints are exchanged with it:

* StaticScore:  log|x| + theta (a learned per-coordinate weight of the magnitude rule);
* ConditionalScore (rank r): log|x| + 1/2 log diag(P^T D(x) P), where D = exp(2 w(x)) with
  w(x) = theta + b tanh(tanh(N(x) E) Dec) and P the RMSNorm Jacobian of the row;
* EvenConditionalScore adds the even feature tanh((N(x) E)^2 - 1) Dec_even;
* ExpandedConditionalScore (rank 64) adds 48 more odd + even features (`extra_*`).

Policy file: {"selected": [{"layer": L, "path": checkpoint}]}; checkpoint file:
{"layer": L, "selected_parameters": {name: nested lists}, ...} (training/models.py:16-52).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from . import LAYERS

NORM_DIM = 512
BOUND = 0.5


def _rms_direction(raw: torch.Tensor, eps: float) -> torch.Tensor:
    return raw * torch.rsqrt(raw.square().mean(-1, keepdim=True) + eps)


def conditional_projected_diagonal(raw: torch.Tensor, log_diagonal: torch.Tensor, eps: float) -> torch.Tensor:
    """diag(P^T D P) for D = diag(exp(log_diagonal)) and P = I - x x^T / (|x|^2 + n eps).

    P is the Jacobian of x -> x / sqrt(mean(x^2) + eps) without its row-uniform scale.  Expanding
    (P^T D P)_ii = d_i - 2 x_i (d_i x_i) / c + x_i^2 sum_j d_j x_j^2 / c^2 with c = |x|^2 + n eps gives
    the closed form below (clamped away from zero for the log).
    """
    if raw.shape != log_diagonal.shape or eps <= 0:
        raise ValueError("one positive diagonal per row and positive epsilon required")
    d = log_diagonal.exp()
    dx = d * raw
    c = raw.square().sum(-1, keepdim=True) + raw.shape[-1] * eps
    quad = (raw * dx).sum(-1, keepdim=True)
    return (d - 2 * raw * dx / c + raw.square() * quad / c.square()).clamp_min(1e-12)


class StaticScore(torch.nn.Module):
    def __init__(self, theta: torch.Tensor):
        super().__init__()
        self.theta = torch.nn.Parameter(theta.detach().clone())

    def forward(self, raw: torch.Tensor, eps: float) -> torch.Tensor:
        return raw.abs().clamp_min(1e-30).log() + self.theta

    def hard_mask(self, ref, raw: torch.Tensor, eps: float) -> torch.Tensor:
        """The kept coordinates: exp of the score, exp(theta) |x|, ranked by the codec's magnitude rule (the same
        order as the scores, ties to the lower coordinate), so a learned static policy packs like TopMag."""
        weighted = torch.exp(self.theta.detach()) * raw.abs()
        return ref.topmag_keep_mask(weighted, 0.5)


class ConditionalScore(torch.nn.Module):
    def __init__(self, theta: torch.Tensor, rank: int = 16, seed: int = 42, residual_bound: float = 0.5):
        super().__init__()
        if theta.shape != (NORM_DIM,) or rank < 1 or not 0 < residual_bound <= 1:
            raise ValueError("512 weights, positive rank and bounded residual required")
        self.theta = torch.nn.Parameter(theta.detach().clone())
        g = torch.Generator(device=theta.device).manual_seed(seed)
        self.encoder = torch.nn.Parameter(
            torch.randn(NORM_DIM, rank, device=theta.device, dtype=theta.dtype, generator=g) / NORM_DIM ** 0.5)
        self.decoder = torch.nn.Parameter(theta.new_zeros(rank, NORM_DIM))
        self.residual_bound = residual_bound

    def log_weights(self, raw: torch.Tensor, eps: float) -> torch.Tensor:
        h = torch.tanh(_rms_direction(raw, eps) @ self.encoder)
        return self.theta + self.residual_bound * torch.tanh(h @ self.decoder)

    def forward(self, raw: torch.Tensor, eps: float) -> torch.Tensor:
        marginal = conditional_projected_diagonal(raw, 2 * self.log_weights(raw, eps), eps)
        return raw.abs().clamp_min(1e-30).log() + 0.5 * marginal.log()


class EvenConditionalScore(ConditionalScore):
    """Adds even (sign-symmetric) features; a zero `decoder_even` reproduces the odd scorer."""

    def __init__(self, theta: torch.Tensor, rank: int = 16, seed: int = 42, residual_bound: float = 0.5):
        super().__init__(theta, rank, seed, residual_bound)
        self.decoder_even = torch.nn.Parameter(theta.new_zeros(rank, NORM_DIM))

    def log_weights(self, raw: torch.Tensor, eps: float) -> torch.Tensor:
        z = _rms_direction(raw, eps) @ self.encoder
        mix = torch.tanh(z) @ self.decoder + torch.tanh(z.square() - 1) @ self.decoder_even
        return self.theta + self.residual_bound * torch.tanh(mix)


class ExpandedConditionalScore(EvenConditionalScore):
    """Rank 16 + 48 features (rank 64); zero `extra_decoder*` reproduce the rank-16 scorer."""

    EXTRA = 48

    def __init__(self, theta: torch.Tensor, seed: int = 42):
        super().__init__(theta, rank=16, seed=seed)
        g = torch.Generator(device=theta.device).manual_seed(seed + 1)
        self.extra_encoder = torch.nn.Parameter(
            torch.randn(NORM_DIM, self.EXTRA, device=theta.device, dtype=theta.dtype, generator=g) / NORM_DIM ** 0.5)
        self.extra_decoder = torch.nn.Parameter(theta.new_zeros(self.EXTRA, NORM_DIM))
        self.extra_decoder_even = torch.nn.Parameter(theta.new_zeros(self.EXTRA, NORM_DIM))

    def log_weights(self, raw: torch.Tensor, eps: float) -> torch.Tensor:
        n = _rms_direction(raw, eps)
        z = n @ self.encoder
        z2 = n @ self.extra_encoder
        mix = (torch.tanh(z) @ self.decoder + torch.tanh(z.square() - 1) @ self.decoder_even
               + torch.tanh(z2) @ self.extra_decoder + torch.tanh(z2.square() - 1) @ self.extra_decoder_even)
        return self.theta + self.residual_bound * torch.tanh(mix)


RANK16_NAMES = {"theta", "encoder", "decoder", "decoder_even"}


class CheckpointError(ValueError):
    """A policy or scorer checkpoint that packmla will not load (the message names the file and the field)."""


def _as_tensor(name: str, value, device=None, dtype=None) -> torch.Tensor:
    try:
        t = torch.as_tensor(value, device=device, dtype=dtype)
    except (TypeError, ValueError) as exc:
        raise CheckpointError(f"parameter {name!r} is not a numeric array") from exc
    if not bool(torch.isfinite(t).all()):
        raise CheckpointError(f"parameter {name!r} holds non-finite values")
    return t


def _check_names(got, want: set, what: str) -> None:
    missing, extra = sorted(want - set(got)), sorted(set(got) - want)
    if missing or extra:
        raise CheckpointError(f"{what}: missing parameters {missing}, unexpected parameters {extra}")


def extend_parameters(parameters: dict, seed: int) -> dict:
    """Rank-16 checkpoint -> rank-64 parameters: the 48 added encoder columns are drawn from `seed`, the added
    decoders are zero, so the extended scorer scores exactly as the rank-16 one did."""
    _check_names(parameters, RANK16_NAMES, "rank-16 warm start")
    model = ExpandedConditionalScore(_as_tensor("theta", parameters["theta"]), seed=seed)
    layout = model.state_dict()
    for name in RANK16_NAMES:
        if tuple(_as_tensor(name, parameters[name]).shape) != tuple(layout[name].shape):
            raise CheckpointError(f"rank-16 warm start: {name!r} has shape "
                                  f"{tuple(torch.as_tensor(parameters[name]).shape)}, expected "
                                  f"{tuple(layout[name].shape)}")
    added = {name: t.tolist() for name, t in layout.items() if name not in RANK16_NAMES}
    return {**parameters, **added}


def initial_rank16_parameters(seed: int) -> dict:
    """A fresh rank-16 scorer (theta 0, decoders 0): scores equal the unweighted conditional rule."""
    m = EvenConditionalScore(torch.zeros(NORM_DIM), rank=16, seed=seed)
    return {k: v.tolist() for k, v in m.state_dict().items()}


def restored_model(parameters: dict, device, seed: int) -> ExpandedConditionalScore:
    """Rank-64 scorer from checkpoint parameters; only theta stays trainable (the evaluation view).

    Every parameter must be present with its shape and finite; theta must lie inside the trust region
    [-BOUND, BOUND] that training keeps it in."""
    template = ExpandedConditionalScore(torch.zeros(NORM_DIM), seed=seed).state_dict()
    _check_names(parameters, set(template), "rank-64 scorer checkpoint")
    loaded = {}
    for name, ref in template.items():
        t = _as_tensor(name, parameters[name], device=device, dtype=ref.dtype)
        if t.shape != ref.shape:
            raise CheckpointError(f"rank-64 scorer checkpoint: {name!r} has shape {tuple(t.shape)}, "
                                  f"expected {tuple(ref.shape)}")
        loaded[name] = t
    if float(loaded["theta"].abs().max()) > BOUND + 1e-7:
        raise CheckpointError(f"rank-64 scorer checkpoint: theta leaves the trust region |theta| <= {BOUND}")
    model = ExpandedConditionalScore(loaded["theta"], seed=seed).to(device)
    model.load_state_dict(loaded)
    for name, p in model.named_parameters():
        p.requires_grad_(name == "theta")
    return model


def _policy_entries(doc, path: Path):
    """The `selected` list of a policy document, or an error naming the file."""
    entries = doc.get("selected") if isinstance(doc, dict) else None
    if not isinstance(entries, list) or len(entries) == 0:
        raise CheckpointError(f"policy {path}: 'selected' must be a non-empty list of {{layer, path}} entries")
    return entries


def read_policy(path: Path, layers: tuple[int, ...] = LAYERS) -> dict[int, dict]:
    """Policy JSON -> {layer: {"layer", "path" (absolute)}}; relative checkpoint paths resolve beside the policy.

    Each entry names one captured layer (a C4 layer index, at most once) and a non-empty checkpoint path."""
    path = Path(path)
    try:
        doc = json.loads(path.read_text())
    except (OSError, json.JSONDecodeError) as exc:
        raise CheckpointError(f"policy {path}: not a readable JSON file") from exc
    table: dict[int, dict] = {}
    for position, entry in enumerate(_policy_entries(doc, path)):
        if not isinstance(entry, dict):
            raise CheckpointError(f"policy {path}: entry {position} is not an object")
        layer, where = entry.get("layer"), entry.get("path")
        if type(layer) is not int or layer not in layers:
            raise CheckpointError(f"policy {path}: entry {position} names layer {layer!r}, not a captured layer")
        if layer in table:
            raise CheckpointError(f"policy {path}: layer {layer} appears twice")
        if not isinstance(where, str) or where == "":
            raise CheckpointError(f"policy {path}: layer {layer} has no checkpoint path")
        target = Path(where) if Path(where).is_absolute() else path.parent / where
        table[layer] = {"layer": layer, "path": str(target.resolve())}
    return table


def read_checkpoint(entry: dict) -> dict:
    """One policy entry's checkpoint record; it must belong to the entry's layer and carry its parameters."""
    path, layer = Path(entry["path"]), entry["layer"]
    try:
        record = json.loads(path.read_text())
    except (OSError, json.JSONDecodeError) as exc:
        raise CheckpointError(f"checkpoint {path} (layer {layer}): not a readable JSON file") from exc
    if not isinstance(record, dict):
        raise CheckpointError(f"checkpoint {path} (layer {layer}): not a JSON object")
    if record.get("layer") != layer:
        raise CheckpointError(f"checkpoint {path}: records layer {record.get('layer')!r}, the policy says {layer}")
    if not isinstance(record.get("selected_parameters"), dict):
        raise CheckpointError(f"checkpoint {path} (layer {layer}): no 'selected_parameters' object")
    return record

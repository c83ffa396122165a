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
        # the magnitude rule on |x| exp(theta): same order as the scores, same tie handling as TopMag
        return ref.topmag_keep_mask(raw.abs() * self.theta.detach().exp(), 0.5)


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


def extend_parameters(parameters: dict, seed: int) -> dict:
    """Rank-16 checkpoint -> rank-64 parameters (new encoder seeded, new decoders zero)."""
    if set(parameters) != RANK16_NAMES:
        raise ValueError("complete rank-16 quadratic warm scorer required")
    model = ExpandedConditionalScore(torch.tensor(parameters["theta"]), seed=seed)
    sd = model.state_dict()
    for name, value in parameters.items():
        if torch.tensor(value).shape != sd[name].shape:
            raise ValueError("warm parameter geometry changed")
    extra = {k: v.tolist() for k, v in sd.items() if k.startswith("extra_")}
    return {**parameters, **extra}


def initial_rank16_parameters(seed: int) -> dict:
    """A fresh rank-16 scorer (theta 0, decoders 0): scores equal the unweighted conditional rule."""
    m = EvenConditionalScore(torch.zeros(NORM_DIM), rank=16, seed=seed)
    return {k: v.tolist() for k, v in m.state_dict().items()}


def restored_model(parameters: dict, device, seed: int) -> ExpandedConditionalScore:
    """Rank-64 scorer from checkpoint parameters; only theta stays trainable (evaluation view)."""
    theta = torch.tensor(parameters["theta"], device=device)
    if theta.shape != (NORM_DIM,) or not bool(torch.isfinite(theta).all()) or float(theta.abs().max()) > BOUND + 1e-7:
        raise ValueError("finite bounded 512 warm weights required")
    model = ExpandedConditionalScore(theta, seed=seed).to(device)
    expected = model.state_dict()
    if set(parameters) != set(expected):
        raise ValueError("complete rank-64 conditional warm model required")
    tensors = {k: torch.as_tensor(v, device=device, dtype=expected[k].dtype) for k, v in parameters.items()}
    for k in expected:
        if tensors[k].shape != expected[k].shape or not bool(torch.isfinite(tensors[k]).all()):
            raise ValueError("warm parameter shape or finiteness changed")
    model.load_state_dict(tensors)
    for name, p in model.named_parameters():
        p.requires_grad_(name == "theta")
    return model


def read_policy(path: Path, layers: tuple[int, ...] = LAYERS) -> dict[int, dict]:
    """Policy JSON -> {layer: {"layer", "path" (absolute)}}; relative paths resolve beside the policy."""
    path = Path(path)
    policy = json.loads(path.read_text())
    entries = policy.get("selected") if isinstance(policy, dict) else None
    if not isinstance(entries, list) or not entries:
        raise ValueError(f"nonempty selected-policy entries required: {path}")
    out: dict[int, dict] = {}
    for e in entries:
        layer = e.get("layer") if isinstance(e, dict) else None
        if type(layer) is not int or layer not in layers or layer in out:
            raise ValueError(f"unique captured policy layers required: {path}: {layer}")
        if not isinstance(e.get("path"), str) or not e["path"]:
            raise ValueError(f"checkpoint path required: {path}: layer {layer}")
        ck = Path(e["path"])
        if not ck.is_absolute():
            ck = path.parent / ck
        out[layer] = {"layer": layer, "path": str(ck.resolve())}
    return out


def read_checkpoint(entry: dict) -> dict:
    path, layer = Path(entry["path"]), entry["layer"]
    try:
        record = json.loads(path.read_text())
    except OSError as exc:
        raise ValueError(f"cannot read policy checkpoint: layer {layer}: {path}") from exc
    if not isinstance(record, dict) or record.get("layer") != layer or not isinstance(
            record.get("selected_parameters"), dict):
        raise ValueError(f"complete selected checkpoint required: layer {layer}")
    return record

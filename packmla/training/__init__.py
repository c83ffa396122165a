"""Offline learned-pruning pipeline: capture -> cache -> fit scorers -> evaluate -> policy.

Same stages, CLI flags and JSON schemas as the reference's `training/` package
(training/__init__.py:7-22, training/train.py:512-534, training/evaluate.py, training/models.py:16-52),
with the reference's external calibration runner replaced by packmla's own fp32 oracle
(packmla.training.calibration): no SGLang checkout is needed.  Capture comes from packmla's model
(packmla.training.data.capture), so the whole loop runs offline on random-init weights.
"""
from __future__ import annotations

# C4 (compress ratio 4) layers of DeepSeek-V4-Flash: the layers whose KV the Packed format prunes.
LAYERS = tuple(range(2, 43, 2))


def parse_layers(text: str, allowed: tuple[int, ...] | None = None) -> tuple[int, ...]:
    """'2,4,8' -> (2, 4, 8); rejects duplicates, unknown layers and empty lists."""
    allowed = LAYERS if allowed is None else allowed
    try:
        layers = tuple(int(x) for x in str(text).split(",") if x.strip())
    except ValueError as exc:
        raise ValueError(f"comma-separated layer ids required: {text!r}") from exc
    if not layers or len(set(layers)) != len(layers) or not set(layers) <= set(allowed):
        raise ValueError(f"unique known C4 layers required: {text!r}")
    return layers

"""CPU: the Native vs Direct format quality check (teacher-forced next-token KL and top-1 agreement)."""
import math

from packmla.bench import quality
from packmla.config import ModelConfig


def test_format_agreement_reports_kl_and_agreement():
    out = quality.main(["--model", "tiny", "--prompts", "2", "--prompt-len", "300", "--steps", "6"])
    assert out["positions"] == 12 and 0.0 <= out["top1_agreement"] <= 1.0
    assert 0.0 <= out["kl_mean"] <= out["kl_max"] and math.isfinite(out["kl_max"])
    assert len(out["first_divergence_step"]) == 2


def test_identical_formats_agree_exactly(monkeypatch):
    """With both engines in the same format the check must report zero divergence (its own control)."""
    real = quality._engine
    monkeypatch.setattr(quality, "_engine", lambda cfg, fmt, *a: real(cfg, "native", *a))
    cfg = ModelConfig.tiny(num_layers=2)
    out = quality.format_agreement(cfg, [[5 + i for i in range(120)]], steps=4)
    assert out["kl_max"] == 0.0 and out["top1_agreement"] == 1.0 and out["first_divergence_step"] == [None]

"""CPU: the offline scorer pipeline (capture -> cache -> fit -> evaluate) and its numerical pieces."""
import json

import pytest
import torch

from packmla.config import ModelConfig
from packmla.training import parse_layers
from packmla.training.calibration import Math, reference
from packmla.training.losses import (BudgetGate, forward_error, forward_errors, packed_rows, preflight,
                                     relaxed_preflight, simulated_packed_rows, stack_states)
from packmla.training.models import (EvenConditionalScore, ExpandedConditionalScore, StaticScore,
                                     conditional_projected_diagonal, extend_parameters, initial_rank16_parameters,
                                     restored_model)


def test_budget_gate_keeps_256_and_is_shift_invariant():
    s = torch.randn(3, 512, dtype=torch.float64, requires_grad=True)
    g = BudgetGate.apply(s, 0.05)
    torch.testing.assert_close(g.sum(-1), torch.full((3,), 256.0, dtype=torch.float64), atol=1e-6, rtol=0)
    c = torch.randn(3, 512, dtype=torch.float64)
    (grad,) = torch.autograd.grad((g * c).sum(), s)
    # the gradient of a common shift of the scores (d/dt of s + t) is zero
    torch.testing.assert_close(grad.sum(-1), torch.zeros(3, dtype=torch.float64), atol=1e-9, rtol=0)


def test_projected_diagonal_matches_explicit_jacobian():
    torch.manual_seed(0)
    x = torch.randn(2, 512, dtype=torch.float64)
    logd = torch.randn(2, 512, dtype=torch.float64) * 0.3
    eps = 1e-6
    got = conditional_projected_diagonal(x, logd, eps)
    for r in range(2):
        c = x[r].square().sum() + 512 * eps
        P = torch.eye(512, dtype=torch.float64) - torch.outer(x[r], x[r]) / c
        ref = torch.diagonal(P.T @ torch.diag(logd[r].exp()) @ P)
        torch.testing.assert_close(got[r], ref.clamp_min(1e-12))


def test_rank16_extension_keeps_scores_and_checkpoint_roundtrip():
    raw = torch.randn(5, 512)
    p16 = initial_rank16_parameters(7)
    p16["theta"] = (torch.rand(512) - 0.5).mul(0.8).tolist()
    p16["decoder"] = (torch.randn(16, 512) * 0.1).tolist()
    m16 = EvenConditionalScore(torch.tensor(p16["theta"]), rank=16, seed=7)
    m16.load_state_dict({k: torch.tensor(v) for k, v in p16.items()})
    p64 = extend_parameters(p16, 7)
    m64 = restored_model(p64, "cpu", 7)
    torch.testing.assert_close(m64(raw, 1e-6), m16(raw, 1e-6))
    assert [n for n, p in m64.named_parameters() if p.requires_grad] == ["theta"]


def _synthetic_state(seed, rows=24, heads=8, swa=16, role="train", rid="a", ordinal=0):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(rows, 512, generator=g) * (torch.rand(512, generator=g) * 3 + 0.1)
    ang = torch.rand(rows, 32, generator=g) * 6.28
    freq = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    weight = torch.rand(512, generator=g) + 0.5
    from packmla.formats import codec

    swa_rows = codec.native_rows(torch.randn(swa, 512, generator=g), weight, 1e-6, freq[:1].expand(swa, -1))
    q = torch.randn(heads, 512, generator=g)
    sink = torch.randn(heads, generator=g)
    qf = freq[0]
    native = codec.native_rows(raw, weight, 1e-6, freq)
    from packmla.training.losses import rounded_output

    out = Math.attention(q, torch.cat((swa_rows, native)), sink, 0.05)[0]
    target = rounded_output(Math, out, qf)
    return {"rid": rid, "ordinal": ordinal, "role": role, "split": role, "raw": raw, "freq": freq, "weight": weight,
            "eps": 1e-6, "q": q, "sink": sink, "scale": 0.05, "swa": swa_rows, "query_freq": qf, "target": target,
            "reference_squared_norm": float(target.square().sum())}


def test_codec_views_and_straight_through_value():
    math, ref = Math(), reference()
    st = _synthetic_state(1)
    model = ExpandedConditionalScore(torch.zeros(512), seed=3)
    mask = torch.ones(24, 512, dtype=torch.bool)
    mask.scatter_(-1, model(st["raw"], 1e-6).topk(256, largest=False).indices, False)
    args = (math, ref, st["raw"], mask, st["weight"], 1e-6, st["freq"])
    assert torch.equal(packed_rows(*args), simulated_packed_rows(*args))
    exact = forward_error(math, ref, st, model)
    ste = forward_error(math, ref, st, model, 0.03)
    assert float(exact) == float(ste) and 0 < float(exact) < 1
    ste.backward()
    assert model.theta.grad is not None and bool(torch.isfinite(model.theta.grad).all())
    # TopMag beats a random static weighting on average: sanity of the error metric
    assert float(forward_error(math, ref, st, StaticScore(torch.zeros(512)))) < 0.5


def test_scalar_and_batched_paths_agree():
    math, ref = Math(), reference()
    states = [_synthetic_state(i, rid=f"r{i}") for i in range(3)]
    model = ExpandedConditionalScore(torch.zeros(512), seed=5)
    with torch.no_grad():
        vec = forward_errors(math, ref, stack_states(states), model)
        sca = torch.stack([forward_error(math, ref, s, model) for s in states])
    torch.testing.assert_close(vec, sca, atol=2e-6, rtol=2e-5)
    assert preflight(math, ref, states, model, 0.02)["states"] == 3
    assert relaxed_preflight(math, states, model, 0.02)["states"] == 3


def test_parse_layers():
    assert parse_layers("2,4") == (2, 4)
    for bad in ("", "3", "2,2", "x"):
        with pytest.raises(ValueError):
            parse_layers(bad)


def test_capture_train_evaluate_end_to_end(tmp_path, monkeypatch):
    from packmla.training import evaluate, train
    from packmla.training.data.cache import load_cached_layer
    from packmla.training.data.capture import capture_cache

    cfg = ModelConfig.tiny(num_layers=2)
    info = capture_cache(tmp_path / "cache", cfg, issues=5, development=2, train_queries=2, dev_queries=2,
                         prompt_len=200)
    layer = cfg.c4_layers[0]
    assert info["states"][layer] == {"train": 6, "development": 4}
    st = load_cached_layer(tmp_path / "cache", layer)
    s0 = st["train"][0]
    assert s0["raw"].shape == (cfg.index_topk, 512) and s0["q"].shape == (cfg.num_heads, 512)
    init = train.main(["--cache", str(tmp_path / "cache"), "--init-policy", str(tmp_path / "init")])
    out = train.main(["--cache", str(tmp_path / "cache"), "--policy", init["policy"], "--output",
                      str(tmp_path / "fit"), "--recipe", "rank64", "--epochs", "2", "--threads", "2"])
    policy = json.loads((tmp_path / "fit" / "policy.json").read_text())
    assert policy["trained_layers"] == [layer] and out["layers"] == [layer]
    # a publish whose linked file is not the staged one is rolled back: no policy.json, progress incomplete
    import os
    import types

    real_stat = os.stat

    def fake_stat(p, *a, **k):
        st = real_stat(p, *a, **k)
        return types.SimpleNamespace(st_ino=st.st_ino + 1) if str(p).endswith("fit2/policy.json") else st

    monkeypatch.setattr(os, "stat", fake_stat)
    with pytest.raises(RuntimeError):
        train.main(["--cache", str(tmp_path / "cache"), "--policy", init["policy"], "--output",
                    str(tmp_path / "fit2"), "--recipe", "rank64", "--epochs", "1", "--threads", "2"])
    monkeypatch.undo()
    assert not (tmp_path / "fit2" / "policy.json").exists()
    assert not (tmp_path / "fit2" / ".policy.json.tmp").exists()
    assert json.loads((tmp_path / "fit2" / "progress.json").read_text())["complete"] is False
    sel = json.loads((tmp_path / "fit" / f"selected-layer-{layer:02d}.json").read_text())
    assert sel["development_selected"]["mean"] <= sel["development_baseline"]["mean"] + 1e-12
    res = evaluate.main(["--cache", str(tmp_path / "cache"), "--policy", out["policy"], "--output",
                         str(tmp_path / "cmp.json"), "--compare-masks"])
    assert {r["method"] for r in res["summary"]} == {"topmag_256", "structured_256", "learned_256", "topmag_192",
                                                     "structured_192", "learned_192"}
    assert (tmp_path / "cmp.md").exists() and (tmp_path / "cmp.csv").exists()
    with pytest.raises(ValueError):  # outputs are never overwritten
        evaluate.main(["--cache", str(tmp_path / "cache"), "--policy", out["policy"], "--output",
                       str(tmp_path / "cmp.json"), "--compare-masks"])
    diag = evaluate.main(["--cache", str(tmp_path / "cache"), "--policy", out["policy"], "--output",
                          str(tmp_path / "diag.json")])
    sweep = evaluate.main(["--cache", str(tmp_path / "cache"), "--policy", out["policy"], "--output",
                           str(tmp_path / "sweep.json"), "--retention-sweep"])
    from packmla.utils.png_plot import read_png

    for metric in ("mean", "p95"):  # curves drawn without matplotlib
        img, text = read_png(tmp_path / f"sweep-{metric}.png")
        assert img.shape == (500, 800, 3) and "topmag=blue" in text["Legend"]
        drawn = [bool((img == c).all(-1).any()) for c in ((31, 119, 180), (255, 127, 14), (44, 160, 44))]
        assert any(drawn)  # curves were drawn (a later series may cover an equal earlier one)
    saved = json.loads((tmp_path / "sweep.json").read_text())
    assert saved["figures"]["renderer"] == "packmla.utils.png_plot" and len(sweep["summary"]) == 21
    from packmla.training.data import storage

    aud = storage.main(["--cache", str(tmp_path / "cache"), "--repeat", "1"])
    lay = aud["layers"][str(layer)]
    assert lay["states"] == {"train": 6, "development": 4}
    assert lay["by_kind"]["raw"] == 10 * cfg.index_topk * 512 * 4 and 0 < lay["tensor_bytes"] <= lay["file_bytes"]
    assert diag["mean_learned"] <= diag["mean_topmag"] * 1.5


def test_capture_cli_writes_fresh_cache(tmp_path):
    from packmla.training.data import capture

    out = capture.main(["--output", str(tmp_path / "c"), "--issues", "2", "--development", "1",
                        "--train-queries", "1", "--dev-queries", "1", "--prompt-len", "64"])
    assert out["skipped"] == 0 and all(v == {"train": 1, "development": 1} for v in out["states"].values())
    with pytest.raises(SystemExit):  # caches are never overwritten
        capture.main(["--output", str(tmp_path / "c")])


def test_capture_cli_publishes_and_builds_from_publications(tmp_path):
    from packmla.training.data import capture, publish
    from packmla.training.data.cache import load_cached_layer

    out = capture.main(["--output", str(tmp_path / "c"), "--publish", str(tmp_path / "pub"), "--issues", "2",
                        "--development", "1", "--train-queries", "1", "--dev-queries", "2", "--prompt-len", "64"])
    cfg = json.loads((tmp_path / "c" / "config.json").read_text())
    assert cfg["model"]["capture_config_sha256"]  # the cache names the configuration it was built from
    issues = sorted(json.loads((tmp_path / "pub" / "capture-config.json").read_text())["requests"])
    reader = publish.PublishedCaptures(tmp_path / "pub", issues)
    layer = out["layers"][0]
    cached = load_cached_layer(tmp_path / "c", layer)
    for role, rows in cached.items():
        for s in rows:
            pub = {p["ordinal"]: p for p in reader.load(s["rid"], layer)}
            assert torch.equal(pub[s["ordinal"]]["target"], s["target"])


def test_png_line_chart_round_trip(tmp_path):
    from packmla.utils.png_plot import line_chart, read_png

    info = line_chart(tmp_path / "c.png", [64, 128, 256], {"a": [1.0, 2.0, 3.5], "b": [0.5, 0.7, 0.9]},
                      title="t", xlabel="x", ylabel="y (%)")
    img, text = read_png(tmp_path / "c.png")
    assert img.shape == (500, 800, 3) and text["Y-Axis"] == "y (%)" and info["legend"] == {"a": "blue", "b": "orange"}
    assert bool((img == (31, 119, 180)).all(-1).any()) and bool((img == (255, 127, 14)).all(-1).any())
    assert info["y_range"][0] <= 0.5 and info["y_range"][1] >= 3.5
    import pytest

    with pytest.raises(FileExistsError):  # never overwrites
        line_chart(tmp_path / "c.png", [1, 2], {"a": [1, 2]})

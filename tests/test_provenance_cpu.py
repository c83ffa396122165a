"""Source gate, run manifests with SHA256SUMS, pinned model profiles (CPU)."""
import hashlib
import json

import pytest

from packmla.utils import model_profiles, provenance


def test_source_identity_reports_the_library_build(tmp_path):
    ident = provenance.source_identity()
    assert ident["csrc_sha256"] and len(ident["csrc_sha256"]) == 64
    assert "library_matches_sources" in ident and "modified" in ident


def test_gate_refuses_a_library_built_from_other_sources(tmp_path, monkeypatch):
    real = provenance.source_identity()
    monkeypatch.setattr(provenance, "source_identity", lambda root=None: {
        **real, "library": {"path": "packmla/_C.so", "sha256": "x", "built_from_sha256": "old"},
        "library_matches_sources": False})
    with pytest.raises(RuntimeError, match="other sources"):
        provenance.check_sources()
    monkeypatch.setattr(provenance, "source_identity", lambda root=None: {
        **real, "library": {"path": "packmla/_C.so", "sha256": "x", "built_from_sha256": real["csrc_sha256"]},
        "library_matches_sources": True, "compiled_modified": ["csrc/attention_decode.cu"]})
    assert provenance.check_sources()["library_matches_sources"]
    with pytest.raises(RuntimeError, match="differ from the commit"):
        provenance.check_sources(strict=True)


def test_sealed_run_verifies_and_detects_changes(tmp_path):
    run = tmp_path / "run-001"
    (run / "raw").mkdir(parents=True)
    (run / "bench.jsonl").write_text('{"value": 1}\n')
    (run / "raw" / "clocks.csv").write_text("a,b\n")
    man = provenance.seal_run(run, ["python", "bench.py"])
    assert man["command"] == ["python", "bench.py"] and man["schema"] == "packmla-run-manifest-v1"
    assert provenance.verify_run(run) == []
    sums = (run / "SHA256SUMS").read_text().splitlines()
    assert any(line.endswith("  raw/clocks.csv") for line in sums)
    with pytest.raises(ValueError, match="already sealed"):
        provenance.seal_run(run)
    (run / "bench.jsonl").write_text('{"value": 2}\n')
    (run / "extra.txt").write_text("x")
    (run / "raw" / "clocks.csv").unlink()
    probs = provenance.verify_run(run)
    assert "changed: bench.jsonl" in probs and "unlisted: extra.txt" in probs and "missing: raw/clocks.csv" in probs


def test_model_profile_verification_is_offline_and_strict(tmp_path, monkeypatch):
    cfg = b'{"model": "fake"}'
    p = model_profiles.ModelProfile("fake", "org/fake", "abc", hashlib.sha256(cfg).hexdigest(), 2, 6,
                                    ("config.json", "model.safetensors.index.json"), None)
    monkeypatch.setitem(model_profiles.PROFILES, "fake", p)
    d = tmp_path / "ckpt"
    d.mkdir()
    (d / "config.json").write_bytes(cfg)
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"a": "s1", "b": "s2", "c": "s1"}}))
    (d / "s1").write_bytes(b"123")
    with pytest.raises(ValueError, match="shards absent"):
        model_profiles.verify_checkpoint("fake", d)
    (d / "s2").write_bytes(b"456")
    assert model_profiles.verify_checkpoint("fake", d, check_bytes=True)["shards"] == 2
    (d / "config.json").write_bytes(b'{"model": "other"}')
    with pytest.raises(ValueError, match="not the pinned"):
        model_profiles.verify_checkpoint("fake", d)
    with pytest.raises(ValueError, match="unknown model family"):
        model_profiles.profile("nope")
    assert model_profiles.profile("dsv4").packmla_config == "v4-flash"

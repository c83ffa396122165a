"""CPU: publication of a trained policy fails closed.  Every injected failure (staging, link,
interrupt, a competing writer, an interrupt after the link) leaves no policy.json of this run and
keeps the finished layers' files; a failed clean-up of the staging name leaves the policy valid."""
import json
import os
from pathlib import Path

import pytest

from packmla.config import ModelConfig
from packmla.training import train
from packmla.training.calibration import Math


@pytest.fixture(scope="module")
def prepared(tmp_path_factory):
    from packmla.training.data.capture import capture_cache

    root = tmp_path_factory.mktemp("publish")
    capture_cache(root / "cache", ModelConfig.tiny(num_layers=2), issues=3, development=1, train_queries=1,
                  dev_queries=1, prompt_len=64)
    init = train.main(["--cache", str(root / "cache"), "--init-policy", str(root / "init")])
    return root, init["policy"]


def _run(root, policy, name):
    return train.main(["--cache", str(root / "cache"), "--policy", policy, "--output", str(root / name),
                       "--recipe", "rank64", "--epochs", "1", "--threads", "2"])


def _fail_stage(monkeypatch):
    real = Math.atomic_json

    def atomic_json(path, obj):
        if Path(path).name == ".policy.json.tmp":
            raise OSError("disk full while staging")
        real(path, obj)

    monkeypatch.setattr(Math, "atomic_json", staticmethod(atomic_json))
    return OSError


def _fail_link(monkeypatch):
    def link(src, dst, *a, **k):
        raise OSError("link refused")

    monkeypatch.setattr(os, "link", link)
    return OSError


def _interrupt_link(monkeypatch):
    def link(src, dst, *a, **k):
        raise KeyboardInterrupt

    monkeypatch.setattr(os, "link", link)
    return KeyboardInterrupt


def _interrupt_after_link(monkeypatch):
    real = os.stat

    def stat(p, *a, **k):
        if str(p).endswith(os.path.join("_interrupt_after_link", "policy.json")):
            raise KeyboardInterrupt
        return real(p, *a, **k)

    monkeypatch.setattr(os, "stat", stat)
    return KeyboardInterrupt


@pytest.mark.parametrize("inject", [_fail_stage, _fail_link, _interrupt_link, _interrupt_after_link])
def test_failed_publication_leaves_no_policy(prepared, monkeypatch, inject):
    root, policy = prepared
    name = inject.__name__
    exc = inject(monkeypatch)
    with pytest.raises(exc):
        _run(root, policy, name)
    monkeypatch.undo()
    out = root / name
    assert not (out / "policy.json").exists() and not (out / ".policy.json.tmp").exists()
    assert json.loads((out / "progress.json").read_text())["complete"] is False
    assert list(out.glob("selected-layer-*.json"))  # finished layers are kept


def test_competing_writer_is_not_overwritten(prepared, monkeypatch):
    root, policy = prepared
    real = os.link

    def link(src, dst, *a, **k):
        Path(dst).write_text('{"competitor": true}')
        return real(src, dst, *a, **k)

    monkeypatch.setattr(os, "link", link)
    with pytest.raises(FileExistsError):
        _run(root, policy, "competitor")
    monkeypatch.undo()
    assert json.loads((root / "competitor" / "policy.json").read_text()) == {"competitor": True}


def test_failed_cleanup_keeps_published_policy(prepared, monkeypatch):
    root, policy = prepared
    real = Path.unlink

    def unlink(self, *a, **k):
        if self.name == ".policy.json.tmp":
            raise OSError("cannot remove staging name")
        return real(self, *a, **k)

    monkeypatch.setattr(Path, "unlink", unlink)
    out = _run(root, policy, "cleanup")
    monkeypatch.undo()
    pub = json.loads(Path(out["policy"]).read_text())
    assert pub["trained_layers"] == out["layers"]
    assert json.loads((root / "cleanup" / "progress.json").read_text())["complete"] is True


def test_cache_rejects_corrupt_incomplete_and_reused(prepared, tmp_path):
    import shutil

    from packmla.training.data.cache import layer_file, load_cached_layer, write_cache

    root, _ = prepared
    layer = json.loads((root / "cache" / "config.json").read_text())["layers"][0]
    assert set(load_cached_layer(root / "cache", layer)) == {"train", "development"}
    bad = tmp_path / "bad"
    shutil.copytree(root / "cache", bad)
    payload = bad / layer_file(layer)
    data = bytearray(payload.read_bytes())
    data[len(data) // 2] ^= 0xFF  # one flipped byte in the middle of the payload
    payload.write_bytes(bytes(data))
    with pytest.raises(ValueError, match="payload changed"):
        load_cached_layer(bad, layer)
    partial = tmp_path / "partial"
    shutil.copytree(root / "cache", partial)
    (partial / "progress.json").write_text(json.dumps({"status": "writing"}))
    with pytest.raises(ValueError, match="complete"):
        load_cached_layer(partial, layer)
    with pytest.raises(ValueError, match="fresh cache directory"):
        write_cache(root / "cache", {}, {"train": [], "development": []}, {})


def test_failed_report_is_rolled_back(prepared, monkeypatch, tmp_path):
    from packmla.training import evaluate

    root, init = prepared
    policy = _run(root, init, "for-report")["policy"]  # evaluation needs a trained rank-64 policy
    real = Math.atomic_json

    def atomic_json(path, obj):
        if Path(path).name == "cmp.json":
            raise KeyboardInterrupt
        real(path, obj)

    monkeypatch.setattr(Math, "atomic_json", staticmethod(atomic_json))
    with pytest.raises(KeyboardInterrupt):
        evaluate.main(["--cache", str(root / "cache"), "--policy", policy, "--output", str(tmp_path / "cmp.json"),
                       "--compare-masks", "--threads", "2"])
    monkeypatch.undo()
    assert sorted(p.name for p in tmp_path.iterdir()) == []  # no partial csv / md / json
    out = evaluate.main(["--cache", str(root / "cache"), "--policy", policy, "--output", str(tmp_path / "cmp.json"),
                         "--compare-masks", "--threads", "2"])
    assert {p.name for p in tmp_path.iterdir()} == {"cmp.json", "cmp.csv", "cmp.md"} and out["summary"]

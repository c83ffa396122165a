"""Published raw captures: verification, bounded reads, cache building and coverage extension (CPU)."""
import json

import pytest
import torch

from packmla.training.data import publish
from packmla.training.data.cache import load_cached_layer

LAYERS = [2, 4]
SPLIT = {"train": ["issue-000", "issue-001"], "development": ["issue-002"], "test": []}


def _state(rid, ordinal, layer, g):
    R, H, W = 6, 4, 3
    target = torch.randn(H, 512, generator=g)
    return {"rid": rid, "ordinal": ordinal, "layer": layer, "raw": torch.randn(R, 512, generator=g),
            "freq": torch.polar(torch.ones(R, 32), torch.rand(R, 32, generator=g)),
            "weight": torch.rand(512, generator=g) + 0.5, "eps": 1e-6, "q": torch.randn(H, 512, generator=g),
            "sink": torch.randn(H, generator=g), "scale": 512 ** -0.5, "swa": torch.randn(W, 512, generator=g),
            "query_freq": torch.polar(torch.ones(32), torch.rand(32, generator=g)), "target": target,
            "reference_squared_norm": float(target.double().square().sum())}


def _publish(root, captured=4):
    g = torch.Generator().manual_seed(0)
    requests = {rid: {"split": role} for role in ("train", "development") for rid in SPLIT[role]}
    publish.write_capture_config(root, {"layers": LAYERS, "split": SPLIT, "requests": requests,
                                        "queries_captured": captured, "model": {"name": "tiny"}})
    for rid in requests:
        publish.publish_issue(root, rid, {layer: [_state(rid, 10 + k, layer, g) for k in range(captured)]
                                          for layer in LAYERS})


def test_publications_build_a_verified_cache(tmp_path):
    _publish(tmp_path / "cap")
    out = publish.build_cache(tmp_path / "cap", tmp_path / "cache", {"train": 2, "development": 3})
    assert out["queries"] == {"train": 2, "development": 3}
    roles = load_cached_layer(tmp_path / "cache", 4)
    assert len(roles["train"]) == 4 and len(roles["development"]) == 3
    assert {s["ordinal"] for s in roles["train"]} == {10, 11}  # the first captured queries, in order
    assert all(s["role"] == "train" for s in roles["train"])


def test_tampered_bundle_is_refused_before_and_after_verification(tmp_path):
    root = tmp_path / "cap"
    _publish(root)
    bundle = root / "bundles" / "issue-001" / "layer-02.pt"
    data = bytearray(bundle.read_bytes())
    data[100] ^= 0xFF
    bundle.write_bytes(bytes(data))
    with pytest.raises(ValueError, match="issue-001"):
        publish.PublishedCaptures(root, ["issue-000", "issue-001"])
    # verified first, changed afterwards: the read refuses it
    root2 = tmp_path / "cap2"
    _publish(root2)
    reader = publish.PublishedCaptures(root2, ["issue-000"])
    f = root2 / "bundles" / "issue-000" / "layer-04.pt"
    f.write_bytes(f.read_bytes())  # same bytes, new file state
    with pytest.raises(ValueError, match="changed after verification"):
        reader.load("issue-000", 4)
    assert reader.load("issue-000", 2)[0]["rid"] == "issue-000"


def test_reads_are_bounded_and_configuration_bound(tmp_path):
    root = tmp_path / "cap"
    _publish(root)
    with pytest.raises(ValueError, match="exceeds"):
        publish.PublishedCaptures(root, ["issue-000"], max_bytes=1000).load("issue-000", 2)
    marker = root / "published" / "issue-002.json"
    rec = json.loads(marker.read_text())
    rec["receipt"]["capture_config_sha256"] = "0" * 64
    marker.write_text(json.dumps(rec))
    with pytest.raises(ValueError, match="another capture configuration"):
        publish.PublishedCaptures(root, ["issue-002"])
    with pytest.raises(ValueError, match="unpublished"):
        (root / "published" / "issue-000.json").unlink()
        publish.PublishedCaptures(root, ["issue-000"])
    with pytest.raises(ValueError, match="already published"):
        publish.publish_issue(root, "issue-001", {})


def test_coverage_extension_keeps_every_original_state(tmp_path):
    root = tmp_path / "cap"
    _publish(root)
    publish.build_cache(root, tmp_path / "base", {"train": 2, "development": 3})
    out = publish.extend_coverage(root, tmp_path / "base", tmp_path / "ext", train_queries=4)
    assert out["added_states"] == 2 * 2 * 2  # 2 issues x 2 queries x 2 layers
    base = load_cached_layer(tmp_path / "base", 2)
    ext = load_cached_layer(tmp_path / "ext", 2)
    assert len(ext["train"]) == 8
    old = {(s["rid"], s["ordinal"]): s for s in base["train"]}
    for s in ext["train"]:
        if (s["rid"], s["ordinal"]) in old:
            assert torch.equal(s["target"], old[(s["rid"], s["ordinal"])]["target"])
    assert [s["ordinal"] for s in ext["development"]] == [s["ordinal"] for s in base["development"]]
    with pytest.raises(ValueError, match="fresh output"):
        publish.extend_coverage(root, tmp_path / "base", tmp_path / "ext", train_queries=4)
    with pytest.raises(ValueError, match="adds training queries"):
        publish.extend_coverage(root, tmp_path / "base", tmp_path / "ext2", train_queries=2)


def test_extension_refuses_a_changed_original(tmp_path):
    root = tmp_path / "cap"
    _publish(root)
    publish.build_cache(root, tmp_path / "base", {"train": 2, "development": 3})
    # republish one issue's bundle with other values under the same names: the verified reader sees the new
    # files, whose first queries no longer match the base cache
    import shutil
    shutil.rmtree(root / "bundles" / "issue-000")
    (root / "published" / "issue-000.json").unlink()
    g = torch.Generator().manual_seed(7)
    publish.publish_issue(root, "issue-000", {layer: [_state("issue-000", 10 + k, layer, g) for k in range(4)]
                                               for layer in LAYERS})
    with pytest.raises(ValueError, match="original training state changed"):
        publish.extend_coverage(root, tmp_path / "base", tmp_path / "ext", train_queries=4)

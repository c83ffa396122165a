"""CPU: GLM-5.3 MLA rows (Native 512 B, Packed 320 B), the Adapter and the decode oracle path."""
import json

import pytest
import torch

from packmla.formats import codec, glm
from packmla.ops.glm import GLMPlanes, glm_packed_to_native, glm_sparse_decode, glm_store


def _rows(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, 512, generator=g), torch.rand(512, generator=g) + 0.5


def test_geometry_and_capacity():
    g = glm.GLM53
    assert g.mla_layers == (3, 7, 11, 15, 19, 23, 27, 31, 35, 39, 43) and g.softmax_scale == 1 / 16
    assert glm.PACKED_ROW_BYTES == 320
    native, direct = glm.bytes_per_token("native"), glm.bytes_per_token("direct")
    assert native == 11 * (512 + 132) and direct == 11 * (320 + 132)
    assert native / direct > 1.4


def test_packed_rows_keep_the_largest_magnitudes_and_renormalize():
    raw, w = _rows(33, 1)
    raw[0] = 0.1
    raw[0, :300] = 1.0  # ties: the lower coordinates win
    values, bitmap = glm.packed_encode(raw, w, 1e-6)
    assert values.shape == (33, 256) and bitmap.shape == (33, 8)
    mask = codec.mask_from_bitmap(bitmap)
    assert torch.equal(mask, codec.topmag_mask(raw, 256))
    assert bool(mask[0, :256].all()) and not bool(mask[0, 256:300].any())
    dense = glm.packed_decode(values, bitmap)
    assert bool((dense[~mask] == 0).all())
    # the kept codes are those of the masked row's Native encoding (the norm runs over the survivors)
    masked_native = glm.native_encode(raw.masked_fill(~mask, 0.0), w, 1e-6)
    assert torch.equal(glm.native_from_packed(values, bitmap)[mask], masked_native[mask])


def test_native_codes_saturate_at_448():
    raw, _ = _rows(4, 2)
    codes = glm.native_encode(raw, torch.full((512,), 1e4), 1e-6)
    dec = glm.native_decode(codes)
    assert bool(torch.isfinite(dec).all()) and float(dec.abs().max()) == 448.0


def test_store_adapter_and_decode_on_cpu():
    raw, w = _rows(40, 3)
    rows = 64
    pool = torch.zeros(rows, 512, dtype=torch.uint8)
    planes = GLMPlanes(torch.zeros(rows, 256, dtype=torch.uint8), torch.zeros(rows, 8, dtype=torch.int64))
    slots = torch.arange(40) + 10
    slots[5] = -1
    glm_store(raw, w, 1e-6, slots, pool=pool)
    glm_store(raw, w, 1e-6, slots, planes=planes)
    keep = slots >= 0
    assert torch.equal(pool[slots[keep]], glm.native_encode(raw[keep], w, 1e-6))
    assert not bool(pool[15].any())  # the skipped row
    nat = glm_packed_to_native(planes, torch.tensor([10, -1, 49, 3]))
    assert torch.equal(nat[0], glm.native_from_packed(planes.values[10:11], planes.bitmap[10:11])[0])
    assert not bool(nat[1].any()) and not bool(nat[3].any())  # a masked row; a row never stored
    assert torch.equal(glm.packed_decode(planes.values[10:11], planes.bitmap[10:11]),
                       glm.native_decode(nat[:1]))

    g = torch.Generator().manual_seed(4)
    B, H, K = 3, 16, 24
    q = torch.randn(B, H, 512, generator=g).bfloat16()
    sl = torch.randint(10, 50, (B, K), generator=g, dtype=torch.int32)
    sl[0, 2] = -1
    lens = torch.tensor([K, 7, 0], dtype=torch.int32)
    for kw in ({"pool": pool}, {"planes": planes}):
        o, lse = glm_sparse_decode(q, sl, lens, **kw)
        ref = []
        for b in range(B):
            s = sl[b, :int(lens[b])].long()
            s = s[s >= 0]
            kv = glm.native_decode(pool[s]) if "pool" in kw else glm.packed_decode(planes.values[s], planes.bitmap[s])
            p = torch.softmax(q[b].float() @ kv.T / 16, -1)
            ref.append(p @ kv if len(s) else torch.zeros(H, 512))
        torch.testing.assert_close(o.float(), torch.stack(ref), atol=1e-2, rtol=1e-2)
        assert bool(torch.isinf(lse[2]).all())  # no rows, no sink


def test_bad_arguments():
    raw, w = _rows(2, 5)
    with pytest.raises(ValueError):
        glm_store(raw, w, 1e-6, torch.arange(2))
    with pytest.raises(ValueError):
        glm.packed_encode(raw, w, 1e-6, mask=torch.ones(2, 512, dtype=torch.bool))


def test_device_batch_limit_is_enforced_before_any_launch():
    from packmla.bench import microbench
    from packmla.ops import glm as glm_ops

    assert glm_ops.MAX_DEVICE_BATCH == 24 and max(microbench.GLM_SUITE_BATCHES) <= glm_ops.MAX_DEVICE_BATCH


def test_suite_record_resumes_only_with_a_matching_manifest(tmp_path):
    from packmla.bench.suite_record import SuiteRecord

    ident = {"csrc_sha256": "a", "library_sha256": "b", "library_built_from": "a"}
    fix = {"suite": "glm", "seed": 1, "rounds": 30}
    out = tmp_path / "glm.jsonl"
    rec = SuiteRecord(out, fix, identity=ident)
    rec.write({"case": "c1", "us": 1.0})
    with pytest.raises(ValueError):
        rec.write({"case": "c1", "us": 2.0})
    with pytest.raises(ValueError, match="exists"):
        SuiteRecord(out, fix, identity=ident)
    with open(out, "a") as f:
        f.write('{"case": "c2", "us"')  # an interrupted write
    again = SuiteRecord(out, fix, resume=True, identity=ident)
    assert again.done == {"c1"}
    again.write({"case": "c2", "us": 3.0})
    assert [json.loads(x)["case"] for x in out.read_text().splitlines()] == ["c1", "c2"]
    with pytest.raises(ValueError, match="library_sha256"):
        SuiteRecord(out, fix, resume=True, identity={**ident, "library_sha256": "other"})
    with pytest.raises(ValueError, match="rounds"):
        SuiteRecord(out, {**fix, "rounds": 10}, resume=True, identity=ident)
    with pytest.raises(ValueError, match="nothing to resume"):
        SuiteRecord(tmp_path / "none.jsonl", fix, resume=True, identity=ident)


def test_glm_pool_lifecycle_capacity_and_decode_on_cpu():
    from packmla.kv.glm_pool import GLMCacheConfig, GLMKVPool, bytes_per_token, capacity_tokens

    for bad in (GLMCacheConfig(kv_cache_format="fp4"), GLMCacheConfig(kv_cache_dtype="bf16"),
                GLMCacheConfig(model_dtype="float16"), GLMCacheConfig(kv_cache_format="direct",
                                                                      enable_hierarchical_cache=True),
                GLMCacheConfig(keep_count=128)):
        with pytest.raises(ValueError):
            GLMKVPool(bad, 4, 2, 256, "cpu")
    native, direct = GLMCacheConfig(), GLMCacheConfig(kv_cache_format="direct")
    assert bytes_per_token(native) == 11 * 644 and bytes_per_token(direct) == 11 * 452
    budget = 64 << 30
    assert capacity_tokens(direct, budget) / capacity_tokens(native, budget) > 1.42
    raw, w = _rows(100, 9)
    g = torch.Generator().manual_seed(10)
    q = torch.randn(1, 16, 512, generator=g).bfloat16()
    outs = {}
    for cfg in (native, direct):
        pool = GLMKVPool(cfg, num_pages=6, max_requests=2, max_context=256, device="cpu")
        slot = pool.admit(100)
        assert pool.pages.free == 4
        pos = torch.arange(100)
        for layer in (3, 43):
            pool.store(layer, raw, w, 1e-6, slot, pos)
        rows = pool.rows_of(slot, pos).int()[None]
        assert pool.rows_of(slot, torch.tensor([200, 256, 1000, -1])).tolist() == [-1] * 4  # no row of its own
        outs[cfg.kv_cache_format] = pool.decode(43, q, rows, torch.tensor([100], dtype=torch.int32))
        pool.release(slot)
        assert pool.pages.free == 6
    # Direct keeps half the coordinates: close to, not equal to, Native
    assert float((outs["native"][0].float() - outs["direct"][0].float()).abs().max()) < 0.5


def test_split_clusters_must_all_be_co_resident(monkeypatch):
    from packmla.ops import attention

    monkeypatch.setitem(attention._MAX_CLUSTERS, 0, {2: 40, 4: 30, 8: 12})
    dev = torch.device("cuda", 0)
    attention.check_cluster_fit(30, 64, 4, dev)  # 30 clusters of 4: co-resident
    attention.check_cluster_fit(500, 128, 9, dev)  # not a cluster count: partials, no limit
    with pytest.raises(ValueError, match="co-resident"):
        attention.check_cluster_fit(32, 16, 4, dev)  # the faulted launch's shape
    with pytest.raises(ValueError, match="co-resident"):
        attention.check_cluster_fit(7, 128, 8, dev)  # 14 clusters of 8 > 12
    # the automatic choice never picks such a count
    assert attention.choose_tiling(32, 16, 2048, max_clusters={2: 40, 4: 30, 8: 12})[0] == 2

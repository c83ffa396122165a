"""CPU: HiCache host tier (write-through of finished requests, restore into a later turn)."""
import pytest
import torch

from packmla.config import EngineConfig, ModelConfig
from packmla.engine.engine import Engine, SamplingParams


def _engine(fmt="direct", hicache=True, pages=None, layout="page_first"):
    from packmla.kv.pool import bytes_per_full_token, fixed_bytes

    cfg = ModelConfig.tiny(num_layers=3)
    ecfg = EngineConfig(kv_cache_format=fmt, device="cpu", chunked_prefill_size=64, max_running_requests=2,
                        cuda_graph_bs=[1, 2], enable_hierarchical_cache=hicache, hicache_ratio=2.0,
                        hicache_mem_layout=layout)
    kv = None
    if pages is not None:
        kv = int(pages * 256 * bytes_per_full_token(cfg, fmt, ecfg.swa_full_tokens_ratio)) + fixed_bytes(cfg, 2) + 4096
    return Engine.build(cfg, ecfg, "cpu", max_context=1024, kv_bytes=kv)


@pytest.mark.parametrize("layout", ["page_first", "layer_first"])
def test_save_restore_round_trip_is_byte_exact(layout):
    for fmt in ("direct", "native"):
        eng = _engine(fmt, layout=layout)
        pool, hc = eng.pool, eng.hicache
        g = torch.Generator().manual_seed(1)
        prompt = torch.randint(3, eng.cfg.vocab_size, (300,), generator=g).tolist()
        eng.generate([prompt], SamplingParams(max_new_tokens=3))
        entry = next(iter(hc.entries.values()))
        assert entry.n_tokens == 302 and len(entry.host_pages) == 2
        # restore into a fresh slot and compare every copied byte with the host copy
        slot = pool.admit(400)
        hc.restore(entry, slot)
        for dev, host in hc._segments(slot, len(entry.host_pages), len(entry.host_c128), entry):
            assert torch.equal(dev, host)
        pool.release(slot)


@pytest.mark.parametrize("layout", ["page_first", "layer_first"])
def test_second_turn_reuses_first_turn_kv(layout):
    g = torch.Generator().manual_seed(2)
    turn1 = torch.randint(3, 512, (260,), generator=g).tolist()
    follow = torch.randint(3, 512, (40,), generator=g).tolist()
    eng = _engine(layout=layout)
    out1 = eng.generate([turn1], SamplingParams(max_new_tokens=4))[0]
    turn2 = turn1 + out1 + follow
    before = eng.metrics.snapshot().get("prefill_tokens", 0)
    out2 = eng.generate([turn2], SamplingParams(max_new_tokens=4))[0]
    m = eng.metrics.snapshot()
    assert m["hicache_hit_tokens"] == len(turn1) + len(out1) - 1
    assert m["prefill_tokens"] - before == len(turn2) - (len(turn1) + len(out1) - 1)
    # same tokens as recomputing turn 2 from scratch (no host tier)
    ref = _engine(hicache=False).generate([turn2], SamplingParams(max_new_tokens=4))[0]
    assert out2 == ref
    eng.flush_cache()
    assert not eng.hicache.entries


def test_lru_eviction_keeps_host_pool_bounded():
    eng = _engine(pages=6)
    hc = eng.hicache
    g = torch.Generator().manual_seed(3)
    for _ in range(12):
        p = torch.randint(3, 512, (500,), generator=g).tolist()
        eng.generate([p], SamplingParams(max_new_tokens=2))
    used = sum(len(e.host_pages) for e in hc.entries.values())
    assert hc.num_host_pages == 12
    assert used <= hc.num_host_pages and hc.stats["evicted"] > 0 and hc.stats["saved"] == 12


def test_layer_first_layout_places_each_plane_in_its_own_region():
    eng = _engine(layout="layer_first")
    hc = eng.hicache
    p0, p1 = hc.planes[0], hc.planes[1]
    assert p0.host_off == 0 and p1.host_off == hc.num_host_pages * p0.page_bytes
    assert hc._host_start(p1, 3, hc.page_bytes) == p1.host_off + 3 * p1.page_bytes
    assert all(hc._host_start(p, h, hc.page_bytes) % 16 == 0 for p in hc.planes for h in range(hc.num_host_pages))
    last = hc.planes[-1]
    assert last.host_off + hc.num_host_pages * last.page_bytes == hc.host.numel()

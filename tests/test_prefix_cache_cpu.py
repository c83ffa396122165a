"""CPU: device prefix cache (finished requests keep their KV slot until the space is needed; a later
prompt that extends one adopts the slot and prefills only its new tokens)."""
import torch

from packmla.config import EngineConfig, ModelConfig
from packmla.engine.engine import Engine, SamplingParams


def _engine(fmt="direct", prefix=True, max_running=2):
    cfg = ModelConfig.tiny(num_layers=3)
    ecfg = EngineConfig(kv_cache_format=fmt, device="cpu", chunked_prefill_size=64, max_running_requests=max_running,
                        cuda_graph_bs=[1, 2, 4], prefix_cache=prefix)
    return Engine.build(cfg, ecfg, "cpu", max_context=1024)


def _toks(n, seed):
    return torch.randint(3, 512, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def test_next_turn_adopts_the_retained_slot_and_matches_recompute():
    for fmt in ("direct", "native"):
        turn1, follow = _toks(300, 1), _toks(37, 2)
        eng = _engine(fmt)
        out1 = eng.generate([turn1], SamplingParams(max_new_tokens=5))[0]
        assert len(eng.retained) == 1
        slot = next(iter(eng.retained.values()))
        turn2 = turn1 + out1 + follow
        before = eng.metrics.snapshot().get("prefill_tokens", 0)
        rid = eng.add_request(turn2, SamplingParams(max_new_tokens=5))
        while eng.has_work():
            eng.step()
        out2 = eng.result(rid).output_ids
        m = eng.metrics.snapshot()
        cached = len(turn1) + len(out1) - 1
        assert m["prefix_cache_hit_tokens"] == cached
        assert m["prefill_tokens"] - before == len(turn2) - cached
        assert eng.result(rid).slot == slot  # the same slot continued
        assert eng.result(rid).cached_tokens == cached
        ref = _engine(fmt, prefix=False).generate([turn2], SamplingParams(max_new_tokens=5))[0]
        assert out2 == ref, fmt


def test_unrelated_prompt_does_not_adopt_and_lru_evicts():
    eng = _engine(max_running=2)
    prompts = [_toks(100, s) for s in (3, 4, 5)]
    outs = [eng.generate([p], SamplingParams(max_new_tokens=3))[0] for p in prompts]
    # two request slots: the third request evicted the least recently used retained slot
    assert len(eng.retained) == 2 and eng.metrics.snapshot()["prefix_cache_evictions"] == 1
    assert tuple(prompts[0] + outs[0][:-1]) not in eng.retained
    ref = _engine(prefix=False)
    assert outs == [ref.generate([p], SamplingParams(max_new_tokens=3))[0] for p in prompts]
    assert not eng.metrics.snapshot().get("prefix_cache_hit_tokens")
    eng.flush_cache()
    assert not eng.retained and eng.pool.pages.free == eng.pool.num_pages


def test_identical_prompt_is_not_a_strict_prefix_and_repeats_exactly():
    eng = _engine()
    p = _toks(80, 7)
    a = eng.generate([p], SamplingParams(max_new_tokens=4))[0]
    b = eng.generate([p], SamplingParams(max_new_tokens=4))[0]
    assert a == b and not eng.metrics.snapshot().get("prefix_cache_hit_tokens")
    assert len(eng.retained) == 1  # the same key replaces its older slot


def test_group_prefills_once_and_copies_match():
    for fmt in ("direct", "native"):
        p = _toks(270, 11)
        eng = _engine(fmt, prefix=False, max_running=4)
        rids = eng.add_group(p, SamplingParams(max_new_tokens=5), n=3)
        while eng.has_work():
            eng.step()
        outs = [eng.result(r).output_ids for r in rids]
        m = eng.metrics.snapshot()
        assert m["prefill_tokens"] == len(p) and m["fork_copied_tokens"] == 2 * len(p)
        ref = _engine(fmt, prefix=False).generate([p], SamplingParams(max_new_tokens=5))[0]
        assert outs == [ref] * 3, fmt  # greedy copies continue exactly like the prefilled request
        assert [eng.result(r).cached_tokens for r in rids] == [0, len(p), len(p)]
        assert eng.pool.pages.free == eng.pool.num_pages


def test_group_without_room_falls_back_to_prefill_and_sampling_is_independent():
    p = _toks(90, 12)
    eng = _engine(prefix=False, max_running=1)  # one running request: the copies wait and prefill alone
    rids = eng.add_group(p, SamplingParams(max_new_tokens=3), n=3)
    while eng.has_work():
        eng.step()
    outs = [eng.result(r).output_ids for r in rids]
    assert outs[0] == outs[1] == outs[2] and eng.metrics.snapshot()["prefill_tokens"] == 3 * len(p)
    eng2 = _engine(prefix=False, max_running=4)
    rids = eng2.add_group(p, SamplingParams(max_new_tokens=6, temperature=1.0), n=4)
    while eng2.has_work():
        eng2.step()
    assert all(len(eng2.result(r).output_ids) == 6 for r in rids)
    # aborting a leader before its prefill hands its copies to ordinary prefill
    eng3 = _engine(prefix=False, max_running=4)
    rids = eng3.add_group(p, SamplingParams(max_new_tokens=2), n=2)
    assert eng3.abort(rids[0])
    while eng3.has_work():
        eng3.step()
    assert len(eng3.result(rids[1]).output_ids) == 2


def _block_engine(max_running=3, fmt="direct", prefix=True, **kw):
    cfg = ModelConfig.tiny(num_layers=3)
    ecfg = EngineConfig(kv_cache_format=fmt, device="cpu", chunked_prefill_size=64, max_running_requests=max_running,
                        cuda_graph_bs=[1, 2, 4], prefix_cache=prefix, prefix_block_tokens=256, **kw)
    return Engine.build(cfg, ecfg, "cpu", max_context=1024)


def test_concurrent_requests_share_prefix_blocks_exactly():
    """Requests submitted together with a shared 512-token prefix: the first prefill caches two 256-token
    blocks (pages by reference, SWA window and pooling states at each block end, the partly filled C128
    page copied); the others map those pages, restore the snapshot and prefill only their own suffix.
    Outputs equal an engine without any prefix cache; every page returns to the pool after a flush."""
    for fmt in ("direct", "native"):
        prefix = _toks(512, 11)
        prompts = [prefix + _toks(40 + 13 * i, 20 + i) for i in range(3)]
        eng = _block_engine(fmt=fmt)
        rids = [eng.add_request(p, SamplingParams(max_new_tokens=5)) for p in prompts]
        while eng.has_work():
            eng.step()
        outs = [eng.result(r).output_ids for r in rids]
        m = eng.metrics.snapshot()
        assert m["prefix_block_hit_tokens"] == 2 * 512, m
        assert m["prefill_tokens"] == sum(len(p) for p in prompts) - 2 * 512
        assert [eng.result(r).cached_tokens for r in rids] == [0, 512, 512]
        assert len(eng.blocks.nodes) == 2
        ref = _block_engine(fmt=fmt, prefix=False)
        assert outs == [ref.generate([p], SamplingParams(max_new_tokens=5))[0] for p in prompts], fmt
        eng.flush_cache()
        assert not eng.blocks.nodes and eng.pool.pages.free == eng.pool.num_pages
        assert eng.pool.c128_pages.free == eng.pool.num_c128_pages


def test_prefix_blocks_chain_and_evict_leaves_first():
    """A longer prompt extends the cached chain (its parent pointer is the last shared block); flushing
    drops retained slots, then the blocks leaves first, and every page returns to the pool."""
    eng = _block_engine(max_running=2)
    base = _toks(512, 31)
    eng.generate([base + _toks(10, 32)], SamplingParams(max_new_tokens=2))
    eng.generate([base + _toks(300, 33)], SamplingParams(max_new_tokens=2))
    assert eng.metrics.snapshot()["prefix_block_hit_tokens"] == 512
    nodes = list(eng.blocks.nodes.values())
    assert sorted(n.index for n in nodes) == [0, 1, 2]
    by_index = {n.index: n for n in nodes}
    assert by_index[2].parent is by_index[1] and by_index[1].parent is by_index[0]
    assert not eng.blocks.evict_one() or len(eng.blocks.nodes) == 2  # a leaf went first
    eng.flush_prefix_cache()
    assert not eng.blocks.nodes and eng.pool.pages.free == eng.pool.num_pages


def test_page_allocator_reference_counts():
    from packmla.kv.pool import PageAllocator

    a = PageAllocator(4)
    p = a.alloc(2)
    a.share(p)
    a.release(p)
    assert a.free == 2  # still held once
    a.release(p)
    assert a.free == 4
    import pytest

    with pytest.raises(ValueError):
        a.release(p)
    with pytest.raises(ValueError):
        a.share(p)


def test_prefix_blocks_with_fp4_and_per_layer_layouts():
    """Shared prefix blocks over FP4 Packed pages and over per-layer Packed survivor counts (read by
    reconstruction) give the tokens of an engine without the cache."""
    cfg = ModelConfig.tiny(num_layers=3)
    counts = {layer: 128 for layer in cfg.c4_layers}
    prefix = _toks(512, 41)
    prompts = [prefix + _toks(30 + 7 * i, 50 + i) for i in range(2)]
    for fmt, kw in (("fp4-direct", {}), ("direct", {"decode_impl": "adapter", "layer_keep_counts": counts})):
        eng = _block_engine(fmt=fmt, **kw)
        rids = [eng.add_request(p, SamplingParams(max_new_tokens=3)) for p in prompts]
        while eng.has_work():
            eng.step()
        assert eng.metrics.snapshot()["prefix_block_hit_tokens"] == 512, fmt
        ref = _block_engine(fmt=fmt, prefix=False, **kw)
        assert [eng.result(r).output_ids for r in rids] == \
            [ref.generate([p], SamplingParams(max_new_tokens=3))[0] for p in prompts], fmt


def test_prefix_blocks_move_to_the_host_tier_and_back():
    """With HiCache on, evicted blocks move to pinned host pages (their KV pages, the C128 pages their
    tokens write, their snapshots) instead of being dropped; a later prompt on the same prefix copies them
    back into new pages, root first, and gives the tokens of an engine without any cache.  With host room
    for one block only, demoting the root drops the host-resident leaf first."""
    prefix = _toks(512, 61)
    first, later = prefix + _toks(33, 62), prefix + _toks(47, 63)
    ref = _block_engine(prefix=False).generate([later], SamplingParams(max_new_tokens=4))[0]
    for ratio, kept in ((2.0, 2), (1e-6, 1)):
        eng = _block_engine(enable_hierarchical_cache=True, hicache_ratio=ratio)
        eng.generate([first], SamplingParams(max_new_tokens=2))
        while eng._evict_retained():
            pass
        eng.hicache.flush()  # only the blocks may serve the later prompt
        while eng.blocks.evict_one():
            pass
        assert eng.blocks.host_nodes == kept and eng.blocks.held_pages == 0
        assert eng.pool.pages.free == eng.pool.num_pages and eng.pool.c128_pages.free == eng.pool.num_c128_pages
        assert eng.blocks.stats["demoted"] == 2 and eng.blocks.stats["dropped"] == 2 - kept
        rid = eng.add_request(later, SamplingParams(max_new_tokens=4))
        while eng.has_work():
            eng.step()
        m = eng.metrics.snapshot()
        assert m["prefix_block_host_hits"] == kept and eng.blocks.host_nodes == 0
        assert eng.result(rid).cached_tokens == 256 * kept
        assert eng.result(rid).output_ids == ref, ratio
        assert eng.server_info()["prefix_blocks_on_host"] == 0
        eng.flush_cache()
        assert not eng.blocks.nodes and eng.pool.pages.free == eng.pool.num_pages
        assert sorted(eng.hicache._free) == list(range(eng.hicache.num_host_pages))


def test_block_under_a_dropped_parent_is_not_cached():
    eng = _block_engine()
    base = _toks(300, 71)
    eng.generate([base], SamplingParams(max_new_tokens=1))
    (node,) = list(eng.blocks.nodes.values())
    while eng._evict_retained():
        pass
    eng.blocks.flush()
    slot = eng.pool.admit(600)
    assert eng.blocks.insert(base + _toks(300, 72), slot, 1, node) is None and not eng.blocks.nodes
    eng.pool.release(slot)
    assert eng.pool.pages.free == eng.pool.num_pages

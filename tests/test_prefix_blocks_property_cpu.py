"""CPU: randomized bookkeeping of the prefix-block tree with the HiCache host tier (no model).

Random admissions on matched chains (promoting host-resident blocks), block insertions, request
releases (some written through to the host tier as request entries, which compete with demoted blocks
for host pages), evictions (demotion to the host or drop) and flushes, with the invariants checked after
every operation: each device page's reference count equals its holders (device blocks and requests),
child counters match the tree, host-resident blocks hold no device pages, host pages are never lost or
doubly owned, and a flush returns every page.
"""
import random
from collections import Counter

import pytest

from packmla.config import EngineConfig, ModelConfig
from packmla.kv.hicache import HostKVCache
from packmla.kv.pool import KVPool
from packmla.kv.prefix_blocks import PrefixBlockCache

BLOCK = 256


def _check(pool, blocks, host, requests):
    pages, c128 = Counter(), Counter()
    for n in blocks.nodes.values():
        if n.host is None:
            pages.update(n.pages)
            c128.update(n.c128_pages)
        else:
            assert n.pages == [] and n.c128_pages == []
    for slot in requests:
        pages.update(pool._req_pages[slot])
        c128.update(pool._req_c128[slot])
    for p in range(pool.num_pages):
        assert pool.pages.refs(p) == pages[p], p
    for p in range(pool.num_c128_pages):
        assert pool.c128_pages.refs(p) == c128[p], p
    assert pool.pages.free == sum(1 for p in range(pool.num_pages) if pages[p] == 0)
    for n in blocks.nodes.values():
        kids = [m for m in blocks.nodes.values() if m.parent is n]
        assert n.children == len(kids) and n.dev_children == sum(m.host is None for m in kids)
        if n.parent is not None:
            assert blocks.nodes.get(n.parent.key) is n.parent  # no orphans
    held = [p for n in blocks.nodes.values() if n.host is not None for p in n.host[0]]
    held += [p for e in host.entries.values() for p in e.host_pages]
    assert sorted(held + host._free) == list(range(host.num_host_pages))
    held128 = [p for n in blocks.nodes.values() if n.host is not None for p in n.host[1]]
    held128 += [p for e in host.entries.values() for p in e.host_c128]
    assert sorted(held128 + host._free_c128) == list(range(host.num_host_c128))


@pytest.mark.parametrize("seed", range(6))
def test_random_block_operations_keep_the_books(seed):
    rng = random.Random(seed)
    cfg = ModelConfig.tiny(num_layers=3)
    pool = KVPool(cfg, EngineConfig(device="cpu", max_running_requests=4), num_pages=24, max_requests=5,
                  max_context=2048, device="cpu")
    host = HostKVCache(pool, ratio=0.4 if seed % 2 else 2.0)
    blocks = PrefixBlockCache(pool, BLOCK)
    blocks.host = host
    prefixes = [[rng.randrange(3, 50) for _ in range(BLOCK * 4)] for _ in range(3)]
    requests: dict[int, dict] = {}
    for _ in range(160):
        op = rng.random()
        if op < 0.35 and pool._free_slots:  # admit on the longest cached chain
            base = rng.choice(prefixes)
            prompt = base[:BLOCK * rng.randint(1, 4)] + [rng.randrange(3, 50) for _ in range(rng.randint(1, 40))]
            chain = blocks.match(prompt)
            need = len(prompt) + 8
            n_sh, n_sh128 = blocks.shared_counts(chain)
            r_pages, r_c128 = blocks.restore_need(chain)
            for n in chain:
                n.pins += 1
            pages_needed = -(-need // BLOCK) - n_sh + r_pages
            c128_needed = -(-need // pool.TOKENS_PER_C128_PAGE) - n_sh128 + r_c128
            while (pages_needed > pool.pages.free or c128_needed > pool.c128_pages.free) and blocks.evict_one():
                pass
            fits = pages_needed <= pool.pages.free and c128_needed <= pool.c128_pages.free
            if fits:
                blocks.promote(chain)
                shared, shared128 = blocks.shared_pages(chain)
                slot = pool.admit(need, shared, shared128)
                if chain:
                    blocks.attach(chain, slot)
                requests[slot] = {"prompt": prompt, "done": len(chain), "tail": chain[-1] if chain else None}
            for n in chain:
                n.pins -= 1
        elif op < 0.65 and requests:  # a request finishes its next block of prefill
            slot = rng.choice(list(requests))
            r = requests[slot]
            if (r["done"] + 1) * BLOCK < len(r["prompt"]):
                r["tail"] = blocks.insert(r["prompt"], slot, r["done"], r["tail"])
                r["done"] += 1
                if r["tail"] is None:  # not cached: later blocks of this request are not either
                    r["done"] = len(r["prompt"])
        elif op < 0.85 and requests:  # a request ends; the host tier may keep its processed tokens
            slot = rng.choice(list(requests))
            r = requests.pop(slot)
            done = min(r["done"] * BLOCK, len(r["prompt"]))
            if done and rng.random() < 0.5:
                host.save(slot, r["prompt"][:done])
            pool.release(slot)
        else:
            blocks.evict_one()
        _check(pool, blocks, host, requests)
    for slot in list(requests):
        pool.release(slot)
    requests.clear()
    assert blocks.stats["demoted"] > 0 and blocks.stats["promoted"] > 0
    blocks.flush()
    host.flush()
    _check(pool, blocks, host, requests)
    assert not blocks.nodes and pool.pages.free == pool.num_pages and pool.c128_pages.free == pool.num_c128_pages

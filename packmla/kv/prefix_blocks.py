"""Prefix sharing between requests in blocks of prompt tokens (8192 by default).

Reference behaviour: SGLang's radix cache, which lets requests that share a prompt prefix (the reference's
generated-shared-prefix workload: a 128k system prompt shared by 40 requests, benchmarks/serving/
shared-prefix-g32-c16-n3-20261020/README.md) reuse its KV pages while they run concurrently.

A request of this model can resume from a prefix only where its whole state is known: the C4 and C128
records before it, the SWA window of the last 128 tokens, and the compressors' pooling state.  At a
multiple of 256 tokens (a KV page) the pending C4 (4-token) and C128 (128-token) groups are empty, and a
request's SWA ring, read at the moment its prefill reaches the boundary, holds exactly the window before
it.  So a block node (default 8192 tokens, the prefill chunk) holds

  * its KV pages (C4 records and indexer keys of every C4 layer), by reference;
  * the C128 pages covering the prefix up to its end, by reference: whole pages (8192 tokens) are shared,
    a partly filled last one is copied into the admitted request's own page (it continues writing there);
  * the SWA ring of every layer at the block's end (a snapshot: 43 layers x 128 Native records, about
    3.2 MB on the V4-Flash geometry) and the compressor / indexer pooling states;

and is keyed by the chain hash of the token blocks up to it.  A request admitted with a matched chain maps
the blocks' pages read-only into its page table (one more page reference each), restores the last
block's snapshot and prefills from there; the records it writes are all past the shared pages.  Nodes are
added as requests finish prefill chunks that end on a block boundary, and evicted least recently used,
leaves first, when the pool needs pages.  A request holds its own page references, so evicting a node
never frees pages a running request reads.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict
from dataclasses import dataclass

import torch

BLOCK_TOKENS = 8192


def _chain_key(parent: bytes, tokens: list[int]) -> bytes:
    h = hashlib.sha256(parent)
    h.update(torch.tensor(tokens, dtype=torch.int64).numpy().tobytes())
    return h.digest()


@dataclass
class BlockNode:
    key: bytes
    parent: "BlockNode | None"
    index: int  # block index: tokens [index * block, (index + 1) * block)
    pages: list[int]  # this block's KV pages
    c128_pages: list[int]  # the C128 pages covering tokens [0, end of this block)
    swa: list[torch.Tensor]  # per layer: the request's ring of W Native records (raw page bytes)
    comp: dict[int, torch.Tensor]
    index_state: dict[int, torch.Tensor]
    children: int = 0
    pins: int = 0  # admissions in progress that matched this node (not evictable meanwhile)
    hits: int = 0


class PrefixBlockCache:
    """Chain-hashed tree of prompt blocks over a KVPool (one per engine rank)."""

    def __init__(self, pool, block_tokens: int = BLOCK_TOKENS):
        if block_tokens <= 0 or block_tokens % pool.TOKENS_PER_PAGE or block_tokens % pool.cfg.window:
            raise ValueError("a block is a whole number of KV pages and of SWA windows")
        self.pool = pool
        self.block = block_tokens
        self.pages_per_block = block_tokens // pool.TOKENS_PER_PAGE
        self.nodes: OrderedDict[bytes, BlockNode] = OrderedDict()  # LRU order (oldest first)

    # ------------------------------------------------------------------ lookup
    def match(self, prompt: list[int]) -> list[BlockNode]:
        """The longest chain of cached blocks that is a prefix of `prompt` and leaves at least one prompt
        token to prefill (its logits start the output)."""
        chain: list[BlockNode] = []
        key = b""
        for i in range((len(prompt) - 1) // self.block):
            key = _chain_key(key, prompt[i * self.block:(i + 1) * self.block])
            node = self.nodes.get(key)
            if node is None:
                break
            chain.append(node)
        return chain

    def shared_pages(self, chain: list[BlockNode]) -> tuple[list[int], list[int]]:
        """(KV pages, whole C128 pages) a request admitted on `chain` maps read-only."""
        pages = [p for n in chain for p in n.pages]
        end = (chain[-1].index + 1) * self.block
        return pages, chain[-1].c128_pages[:end // self.pool.TOKENS_PER_C128_PAGE]

    def attach(self, chain: list[BlockNode], slot: int) -> None:
        """A request admitted on `chain` (its pages already mapped): copy the partly filled C128 page and
        restore the last block's SWA window and pooling states into its slot."""
        pool = self.pool
        last = chain[-1]
        end = (last.index + 1) * self.block
        full = end // pool.TOKENS_PER_C128_PAGE
        if end % pool.TOKENS_PER_C128_PAGE:  # the partly filled C128 page: a private copy
            src, dst = last.c128_pages[full], pool._req_c128[slot][full]
            for t in pool.c128_native.values():
                pages = t.view(pool.num_c128_pages, -1)
                pages[dst].copy_(pages[src])
        for layer, ring in enumerate(last.swa):
            pool.swa[layer].view(pool.max_requests, -1)[slot].copy_(ring)
        for layer, st in last.comp.items():
            pool.comp_state[layer][slot].copy_(st)
        for layer, st in last.index_state.items():
            pool.index_state[layer][slot].copy_(st)
        for n in chain:
            n.hits += 1
            self.nodes.move_to_end(n.key)

    # ------------------------------------------------------------------ insertion
    def insert(self, prompt: list[int], slot: int, index: int, parent: BlockNode | None) -> BlockNode | None:
        """Block `index` of `prompt` has just been prefilled by the request in `slot` (its prefill is at the
        block's end): add it, or find the same block already cached.  Returns the node (None: not cached)."""
        if (parent is None) != (index == 0):
            return None
        key = _chain_key(parent.key if parent else b"", prompt[index * self.block:(index + 1) * self.block])
        node = self.nodes.get(key)
        if node is not None:
            self.nodes.move_to_end(key)
            return node
        pool = self.pool
        end = (index + 1) * self.block
        n128 = -(-end // pool.TOKENS_PER_C128_PAGE)
        pages = pool._req_pages[slot][index * self.pages_per_block:(index + 1) * self.pages_per_block]
        c128 = pool._req_c128[slot][:n128]
        if len(pages) != self.pages_per_block or len(c128) != n128:
            return None
        node = BlockNode(key, parent, index, list(pages), list(c128),
                         [t.view(pool.max_requests, -1)[slot].clone() for t in pool.swa],
                         {l: st[slot].clone() for l, st in pool.comp_state.items()},
                         {l: st[slot].clone() for l, st in pool.index_state.items()})
        pool.pages.share(node.pages)
        pool.c128_pages.share(node.c128_pages)
        if parent is not None:
            parent.children += 1
        self.nodes[key] = node
        return node

    # ------------------------------------------------------------------ eviction
    def evict_one(self) -> bool:
        """Drop the least recently used block that no admission holds and no block extends."""
        for node in self.nodes.values():
            if node.children == 0 and node.pins == 0:
                self._drop(node)
                return True
        return False

    def _drop(self, node: BlockNode) -> None:
        del self.nodes[node.key]
        self.pool.pages.release(node.pages)
        self.pool.c128_pages.release(node.c128_pages)
        if node.parent is not None:
            node.parent.children -= 1

    def flush(self) -> None:
        """Drop every block (leaves first)."""
        while self.evict_one():
            pass

    @property
    def held_pages(self) -> int:
        return sum(len(n.pages) for n in self.nodes.values())

    def snapshot_bytes(self) -> int:
        return sum(sum(t.numel() * t.element_size() for t in n.swa) for n in self.nodes.values())

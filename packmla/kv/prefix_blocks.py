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

Host tier (with HiCache on, as SGLang's hierarchical radix cache demotes evicted radix nodes to host
memory): an evicted node whose extensions are all host-resident moves to pinned host pages instead of
being dropped: its own KV pages, the C128 pages its token range writes (the first one, when the block
starts inside a C128 page, also holds the parent's records, identical in every copy) and its snapshot.
A match that reaches host-resident nodes copies them back into freshly allocated pages, root first, and
rebuilds each node's C128 list as its parent's whole pages followed by its own.  Host room is made by
dropping host-resident leaves, then HiCache's request entries; a node that finds none is dropped with its
descendants.
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
    dev_children: int = 0  # children whose pages are on the device
    pins: int = 0  # admissions in progress that matched this node (not evictable meanwhile)
    hits: int = 0
    host: tuple | None = None  # (host pages, host C128 pages) while the node lives in the host tier


def _to_host(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cuda":
        return t
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t, non_blocking=True)  # ordered before any later reuse of `t`'s memory on this stream
    return h


class PrefixBlockCache:
    """Chain-hashed tree of prompt blocks over a KVPool (one per engine rank)."""

    def __init__(self, pool, block_tokens: int = BLOCK_TOKENS):
        if block_tokens <= 0 or block_tokens % pool.TOKENS_PER_PAGE or block_tokens % pool.cfg.window:
            raise ValueError("a block is a whole number of KV pages and of SWA windows")
        self.pool = pool
        self.block = block_tokens
        self.pages_per_block = block_tokens // pool.TOKENS_PER_PAGE
        self.nodes: OrderedDict[bytes, BlockNode] = OrderedDict()  # LRU order (oldest first)
        self.host = None  # a HostKVCache: evicted blocks move there instead of being dropped
        self.stats = {"demoted": 0, "promoted": 0, "dropped": 0}

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

    def shared_counts(self, chain: list[BlockNode]) -> tuple[int, int]:
        """How many (KV pages, C128 pages) a request admitted on `chain` maps instead of allocating."""
        if not chain:
            return 0, 0
        end = (chain[-1].index + 1) * self.block
        return len(chain) * self.pages_per_block, end // self.pool.TOKENS_PER_C128_PAGE

    def shared_pages(self, chain: list[BlockNode]) -> tuple[list[int], list[int]]:
        """(KV pages, whole C128 pages) a request admitted on `chain` maps read-only (all on the device)."""
        if not chain:
            return [], []
        if any(n.host is not None for n in chain):
            raise ValueError("host-resident blocks must be promoted before they are mapped")
        pages = [p for n in chain for p in n.pages]
        return pages, chain[-1].c128_pages[:self.shared_counts(chain)[1]]

    # ------------------------------------------------------------------ host tier
    def _own_c128(self, node: BlockNode) -> tuple[int, int]:
        """[first, end) of the C128 pages that tokens of `node`'s block are written to."""
        c = self.pool.TOKENS_PER_C128_PAGE
        return node.index * self.block // c, -(-(node.index + 1) * self.block // c)

    def restore_need(self, chain: list[BlockNode]) -> tuple[int, int]:
        """Device (KV pages, C128 pages) that promoting the host-resident nodes of `chain` allocates."""
        pages = c128 = 0
        for n in chain:
            if n.host is not None:
                first, end = self._own_c128(n)
                pages += self.pages_per_block
                c128 += end - first
        return pages, c128

    def promote(self, chain: list[BlockNode]) -> int:
        """Copy the host-resident nodes of `chain` back to the device (root first; the pool has the pages).
        Returns how many were promoted."""
        count = 0
        for node in chain:
            if node.host is None:
                continue
            pool = self.pool
            hp, h128 = node.host
            first, _ = self._own_c128(node)
            pages, own128 = pool.pages.alloc(len(hp)), pool.c128_pages.alloc(len(h128))
            self.host.copy_pages(pages, hp, own128, h128, to_host=False)
            base = node.parent.c128_pages[:first] if node.parent is not None else []
            pool.c128_pages.share(base)
            node.pages, node.c128_pages = pages, list(base) + own128
            dev = pool.device
            node.swa = [t.to(dev, non_blocking=True) for t in node.swa]
            node.comp = {l: t.to(dev, non_blocking=True) for l, t in node.comp.items()}
            node.index_state = {l: t.to(dev, non_blocking=True) for l, t in node.index_state.items()}
            self.host.free_host(hp, h128)  # later writes to these host pages queue behind this copy
            node.host = None
            if node.parent is not None:
                node.parent.dev_children += 1
            self.stats["promoted"] += 1
            count += 1
        return count

    def _host_room(self, n_pages: int, n_c128: int) -> tuple | None:
        got = self.host.alloc_host(n_pages, n_c128, evict_entries=False)
        while got is None:
            leaf = next((n for n in self.nodes.values()
                         if n.host is not None and n.children == 0 and n.pins == 0), None)
            if leaf is None:
                return self.host.alloc_host(n_pages, n_c128, evict_entries=True)
            self._drop(leaf)
            got = self.host.alloc_host(n_pages, n_c128, evict_entries=False)
        return got

    def _demote(self, node: BlockNode) -> bool:
        first, _ = self._own_c128(node)
        own128 = node.c128_pages[first:]
        got = self._host_room(len(node.pages), len(own128))
        if got is None:
            return False
        hp, h128 = got
        self.host.copy_pages(node.pages, hp, own128, h128, to_host=True)
        node.swa = [_to_host(t) for t in node.swa]
        node.comp = {l: _to_host(t) for l, t in node.comp.items()}
        node.index_state = {l: _to_host(t) for l, t in node.index_state.items()}
        self.pool.pages.release(node.pages)
        self.pool.c128_pages.release(node.c128_pages)
        node.pages, node.c128_pages, node.host = [], [], (hp, h128)
        if node.parent is not None:
            node.parent.dev_children -= 1
        self.stats["demoted"] += 1
        return True

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
        if parent is not None and self.nodes.get(parent.key) is not parent:
            return None  # the parent was dropped since: a block under it could never be matched
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
            parent.dev_children += 1
        self.nodes[key] = node
        return node

    # ------------------------------------------------------------------ eviction
    def evict_one(self) -> bool:
        """Free the device pages of the least recently used block that no admission holds and no
        device-resident block extends: move it to the host tier when there is one with room, else drop it
        (with its descendants, which resume from it)."""
        for node in self.nodes.values():
            if node.host is None and node.dev_children == 0 and node.pins == 0:
                if self.host is None or not self._demote(node):
                    self._drop(node)
                return True
        return False

    def _drop(self, node: BlockNode) -> None:
        for child in [n for n in self.nodes.values() if n.parent is node]:
            self._drop(child)
        del self.nodes[node.key]
        if node.host is None:
            self.pool.pages.release(node.pages)
            self.pool.c128_pages.release(node.c128_pages)
        else:
            self.host.free_host(*node.host)
        if node.parent is not None:
            node.parent.children -= 1
            if node.host is None:
                node.parent.dev_children -= 1
        self.stats["dropped"] += 1

    def flush(self) -> None:
        """Drop every block, device- and host-resident."""
        for root in [n for n in self.nodes.values() if n.parent is None]:
            self._drop(root)

    @property
    def held_pages(self) -> int:
        return sum(len(n.pages) for n in self.nodes.values())

    @property
    def host_nodes(self) -> int:
        return sum(n.host is not None for n in self.nodes.values())

    def snapshot_bytes(self) -> int:
        """Device bytes of the SWA snapshots of device-resident blocks."""
        return sum(sum(t.numel() * t.element_size() for t in n.swa)
                   for n in self.nodes.values() if n.host is None)

"""HiCache: a pinned host tier for the KV of finished requests, restored when a later prompt extends them.

Reference behaviour (SGLang HiCache as the reference configures it: `--enable-hierarchical-cache`,
`--hicache-ratio 2.0`, page-first layout, write-through, kernel IO backend; Packed support moves the
value, bitmap and scale planes of a page together, 256-survivor layout only — third_party/README.md
:190, :261, scripts/local/run-server.sh:134-139).  packmla's engine keeps KV per request, so the host
tier works at request granularity: when a request finishes, its KV (every C4 page of every C4 layer
with all planes and indexer keys, its C128 pages, and the request slot's SWA ring and compressor
state) is written through to host memory, keyed by the processed tokens.  A new request whose prompt
starts with such a key gets the KV copied back into its freshly allocated pages and prefills only the
remaining tokens (a multi-turn conversation re-sends its history every turn).  The same host pages also
hold prefix blocks evicted from the device block tree (`packmla.kv.prefix_blocks`): `alloc_host` /
`copy_pages` / `free_host` move a block's own KV and C128 pages, and a block may take the pages of
least recently used request entries, never the reverse.

Layout: `page_first` (default: one host page holds the page's planes of all layers contiguously, so a
request's pages are few large segments) or `layer_first` (each plane of each layer has its own host
region indexed by host page, as SGLang's layer-first host pool); `ratio` x the device page count host
pages exist; entries are evicted least-recently-used.  Moves are
one `segment_copy` kernel launch per direction on a side stream (pinned host memory is device-mapped);
on CPU pools the same segments are plain tensor copies.
"""
from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

from ..formats import abi
from .pool import KVPool

_Q = 16  # every segment is 16-byte aligned with a size that is a multiple of 16


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8).reshape(-1)


@dataclass
class Entry:
    tokens: tuple
    n_tokens: int
    host_pages: list[int]
    host_c128: list[int]
    slot_state: torch.Tensor
    hits: int = 0


@dataclass
class _Plane:
    """One per-page plane of one layer: device byte view, bytes per page, offset inside a host page."""
    dev: torch.Tensor
    page_bytes: int
    host_off: int = 0


class HostKVCache:
    def __init__(self, pool: KVPool, ratio: float = 2.0, layout: str = "page_first"):
        if pool.kv_format == "direct" and pool.ecfg.keep_count != abi.PACKED_KEEP:
            raise ValueError("HiCache requires the 256-survivor layout")
        if layout not in ("page_first", "layer_first"):
            raise ValueError("HiCache layout must be page_first or layer_first")
        self.layout = layout
        self.pool = pool
        self.dev = pool.device
        R = abi.RECORDS_PER_PAGE
        planes: list[_Plane] = []
        for layer in pool.cfg.c4_layers:
            if pool.kv_format == "direct":
                planes += [_Plane(_bytes(pool.c4_values[layer]), R * abi.PACKED_KEEP),
                           _Plane(_bytes(pool.c4_bitmap[layer]), R * abi.BITMAP_WORDS * 8),
                           _Plane(_bytes(pool.c4_scales[layer]), R * abi.NUM_TILES)]
            else:
                planes.append(_Plane(_bytes(pool.c4_native[layer]), abi.NATIVE_PAGE_BYTES))
            planes += [_Plane(_bytes(pool.index_keys[layer]), R * pool.cfg.index_dim),
                       _Plane(_bytes(pool.index_scales[layer]), R * 4)]
        off = 0
        for p in planes:
            if p.page_bytes % _Q:
                raise ValueError("page planes must be multiples of 16 bytes")
            p.host_off = off
            off += p.page_bytes
        self.planes = planes
        self.page_bytes = off
        self.c128_planes = [_Plane(_bytes(t), abi.NATIVE_PAGE_BYTES) for t in pool.c128_native.values()]
        off = 0
        for p in self.c128_planes:
            p.host_off = off
            off += p.page_bytes
        self.c128_page_bytes = off
        # per-slot state: SWA ring pages of every layer + compressor / indexer pooling state
        self.swa_slot_bytes = (pool.cfg.window // abi.RECORDS_PER_PAGE) * abi.NATIVE_PAGE_BYTES
        self.state_tensors = list(pool.comp_state.values()) + list(pool.index_state.values())
        self.slot_state_bytes = (pool.cfg.num_layers * self.swa_slot_bytes
                                 + sum(t[0].numel() * 4 for t in self.state_tensors))
        self.num_host_pages = max(1, math.ceil(ratio * pool.num_pages))
        self.num_host_c128 = max(1, math.ceil(ratio * pool.num_c128_pages))
        if layout == "layer_first":  # plane regions: region start = host_off x number of host pages
            for p in self.planes:
                p.host_off *= self.num_host_pages
            for p in self.c128_planes:
                p.host_off *= self.num_host_c128
        pin = self.dev.type == "cuda"
        self.host = torch.zeros(self.num_host_pages * self.page_bytes, dtype=torch.uint8, pin_memory=pin)
        self.host_c128 = torch.zeros(max(1, self.num_host_c128 * self.c128_page_bytes), dtype=torch.uint8,
                                     pin_memory=pin)
        self._free = list(range(self.num_host_pages - 1, -1, -1))
        self._free_c128 = list(range(self.num_host_c128 - 1, -1, -1))
        self.entries: "OrderedDict[tuple, Entry]" = OrderedDict()
        self.stream = torch.cuda.Stream(self.dev) if pin else None
        self.stats = {"saved": 0, "restored": 0, "restored_tokens": 0, "evicted": 0, "bytes_d2h": 0, "bytes_h2d": 0}

    # ------------------------------------------------------------------ segments
    def _segments(self, slot: int, n_pages: int, n_c128: int, entry: Entry) -> list[tuple]:
        """(device view, host view) pairs of one request's KV, in host-page order."""
        pool = self.pool
        pairs = []
        for i in range(n_pages):
            dpage = pool._req_pages[slot][i]
            for p in self.planes:
                h = self._host_start(p, entry.host_pages[i], self.page_bytes)
                pairs.append((p.dev[dpage * p.page_bytes:(dpage + 1) * p.page_bytes],
                              self.host[h:h + p.page_bytes]))
        for i in range(n_c128):
            dpage = pool._req_c128[slot][i]
            for p in self.c128_planes:
                h = self._host_start(p, entry.host_c128[i], self.c128_page_bytes)
                pairs.append((p.dev[dpage * p.page_bytes:(dpage + 1) * p.page_bytes],
                              self.host_c128[h:h + p.page_bytes]))
        off = 0
        for swa in pool.swa:
            b = _bytes(swa)
            pairs.append((b[slot * self.swa_slot_bytes:(slot + 1) * self.swa_slot_bytes],
                          entry.slot_state[off:off + self.swa_slot_bytes]))
            off += self.swa_slot_bytes
        for t in self.state_tensors:
            row = _bytes(t[slot])
            pairs.append((row, entry.slot_state[off:off + row.numel()]))
            off += row.numel()
        return pairs

    def _host_start(self, p: _Plane, host_page: int, page_bytes: int) -> int:
        """Byte offset of plane `p` of `host_page` in the host buffer."""
        if self.layout == "layer_first":
            return p.host_off + host_page * p.page_bytes
        return host_page * page_bytes + p.host_off

    def _run(self, pairs: list[tuple], to_host: bool) -> int:
        if any(d.numel() != h.numel() for d, h in pairs):  # a clipped view would make the kernel overrun
            raise ValueError("HiCache segment views differ in size")
        nbytes = sum(d.numel() for d, _ in pairs)
        if self.stream is None:
            for d, h in pairs:
                (h if to_host else d).copy_(d if to_host else h)
            return nbytes
        from ..ops._ext import ext

        segs = torch.tensor([[d.data_ptr(), h.data_ptr(), d.numel()] if to_host else
                             [h.data_ptr(), d.data_ptr(), d.numel()] for d, h in pairs], dtype=torch.int64)
        if any(int(x) % _Q for row in segs.tolist() for x in row):
            raise ValueError("HiCache segments must be 16-byte aligned")
        main = torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(main)  # the KV being saved / the pages being filled are ordered after compute
        with torch.cuda.stream(self.stream):
            segs_d = segs.pin_memory().to(self.dev, non_blocking=True)
            ext().segment_copy(segs_d)
            segs_d.record_stream(self.stream)
        main.wait_stream(self.stream)  # the next forward may read restored pages; pages may be reused
        return nbytes

    # ------------------------------------------------------------------ host allocation
    def _evict_until(self, pages: int, c128: int) -> bool:
        while (len(self._free) < pages or len(self._free_c128) < c128) and self.entries:
            _, old = self.entries.popitem(last=False)
            self._free.extend(old.host_pages)
            self._free_c128.extend(old.host_c128)
            self.stats["evicted"] += 1
        return len(self._free) >= pages and len(self._free_c128) >= c128

    # ------------------------------------------------------------------ public
    def save(self, slot: int, tokens: list[int]) -> Entry | None:
        """Write through the KV of `tokens` (all processed by the model) held by request `slot`."""
        n = len(tokens)
        if n == 0:
            return None
        key = tuple(tokens)
        if key in self.entries:
            self.entries.move_to_end(key)
            return self.entries[key]
        n_pages = -(-n // KVPool.TOKENS_PER_PAGE)
        n_c128 = -(-n // KVPool.TOKENS_PER_C128_PAGE)
        if (n_pages > len(self.pool._req_pages[slot]) or n_c128 > len(self.pool._req_c128[slot])
                or n_pages > self.num_host_pages or n_c128 > self.num_host_c128):
            return None
        if not self._evict_until(n_pages, n_c128):
            return None
        entry = Entry(key, n, [self._free.pop() for _ in range(n_pages)], [self._free_c128.pop() for _ in range(n_c128)],
                      torch.zeros(self.slot_state_bytes, dtype=torch.uint8, pin_memory=self.stream is not None))
        self.stats["bytes_d2h"] += self._run(self._segments(slot, n_pages, n_c128, entry), to_host=True)
        self.entries[key] = entry
        self.stats["saved"] += 1
        return entry

    def match(self, prompt: list[int]) -> Entry | None:
        """Longest saved context that is a strict prefix of `prompt` (at least one token left to prefill)."""
        best = None
        for key, e in self.entries.items():
            if e.n_tokens < len(prompt) and (best is None or e.n_tokens > best.n_tokens) and \
                    tuple(prompt[:e.n_tokens]) == key:
                best = e
        return best

    def restore(self, entry: Entry, slot: int) -> int:
        """Copy `entry` into request `slot` (pages already allocated for the whole request)."""
        n_pages = len(entry.host_pages)
        n_c128 = len(entry.host_c128)
        self.stats["bytes_h2d"] += self._run(self._segments(slot, n_pages, n_c128, entry), to_host=False)
        entry.hits += 1
        self.entries.move_to_end(entry.tokens)
        self.stats["restored"] += 1
        self.stats["restored_tokens"] += entry.n_tokens
        return entry.n_tokens

    def flush(self) -> None:
        for e in self.entries.values():
            self._free.extend(e.host_pages)
            self._free_c128.extend(e.host_c128)
        self.entries.clear()

    # ------------------------------------------------------------------ page lists (prefix blocks)
    def alloc_host(self, n_pages: int, n_c128: int, evict_entries: bool = True) -> tuple | None:
        """Host pages for a prefix block's pages (request entries are evicted first when `evict_entries`)."""
        if evict_entries:
            self._evict_until(n_pages, n_c128)
        if len(self._free) < n_pages or len(self._free_c128) < n_c128:
            return None
        return [self._free.pop() for _ in range(n_pages)], [self._free_c128.pop() for _ in range(n_c128)]

    def free_host(self, host_pages: list[int], host_c128: list[int]) -> None:
        self._free.extend(host_pages)
        self._free_c128.extend(host_c128)

    def copy_pages(self, dev_pages: list[int], host_pages: list[int], dev_c128: list[int], host_c128: list[int],
                   to_host: bool) -> int:
        """Every plane of the given device pages <-> the given host pages, in one segment-copy launch."""
        pairs = []
        for d, h in zip(dev_pages, host_pages):
            for p in self.planes:
                o = self._host_start(p, h, self.page_bytes)
                pairs.append((p.dev[d * p.page_bytes:(d + 1) * p.page_bytes], self.host[o:o + p.page_bytes]))
        for d, h in zip(dev_c128, host_c128):
            for p in self.c128_planes:
                o = self._host_start(p, h, self.c128_page_bytes)
                pairs.append((p.dev[d * p.page_bytes:(d + 1) * p.page_bytes], self.host_c128[o:o + p.page_bytes]))
        n = self._run(pairs, to_host) if pairs else 0
        self.stats["bytes_d2h" if to_host else "bytes_h2d"] += n
        return n

    def host_bytes(self) -> int:
        return self.host.numel() + self.host_c128.numel()

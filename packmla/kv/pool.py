"""Paged KV memory for compressed-sparse MLA layers, with capacity accounting.

Layout (per rank; the latent KV is shared by all heads, so TP ranks hold full copies):

* page = 256 tokens = 64 C4 records.  A request owns a row of the page table; the same
  page id addresses every C4 layer's pool (one allocation serves all layers).
* C4 layers:   Native pages (584 B/record) in `native` mode, or Packed planes
               (256 + 64 + 8 B/record) in `direct` mode, or FP4 pages (288 B / 224 B per record, data
               rows then scale rows) in `fp4-native` / `fp4-direct` mode; plus FP8 indexer keys
               (index_dim B + 4 B fp32 scale per record).
* C128 layers: Native pages; one C128 record per 128 tokens, 64 records per C128 page.
* SWA:         per layer a ring of 128 Native records per request slot.
* compressor state: online-softmax pooling state (max, sum, weighted sum) per layer per
  request slot for the latent (512) and, on C4 layers, the indexer key.

Capacity follows the reference's accounting (`DSV4 memory calculation: bytes_per_full_token`
in the serve logs): bytes per full token = C4 record bytes / 4 over C4 layers + indexer key
bytes / 4 + C128 record bytes / 128 + swa_full_tokens_ratio x SWA bytes over all layers.
The Packed/Native ratio of `max_total_tokens` is the KV-capacity metric (reference: 1.2113x,
docs/report.md:30).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..config import EngineConfig, ModelConfig
from ..formats import abi, fp4


@dataclass
class CapacityReport:
    kv_format: str
    bytes_per_full_token: float
    available_bytes: int
    fixed_bytes: int
    max_total_tokens: int
    num_pages: int

    def as_dict(self) -> dict:
        return dict(self.__dict__)


def c4_record_bytes(kv_format: str, keep: int = abi.PACKED_KEEP) -> int:
    """Logical bytes of one C4 record; a Packed record with K survivors is K + 72 bytes."""
    if kv_format.startswith("fp4-"):
        return fp4.record_bytes(kv_format[4:])
    return keep + abi.BITMAP_WORDS * 8 + abi.NUM_TILES if kv_format == "direct" else abi.NATIVE_RECORD_BYTES


def bytes_per_full_token(cfg: ModelConfig, kv_format: str, swa_ratio: float,
                         keep_for=None) -> float:
    """`keep_for(layer)`: a C4 layer's Packed survivor count (default 256 everywhere); the layers' actual
    record sizes are summed, smaller layouts are not padded."""
    c4 = sum(c4_record_bytes(kv_format, keep_for(layer) if keep_for else abi.PACKED_KEEP) + cfg.index_dim + 4
             for layer in cfg.c4_layers) / abi.C4_RATIO
    c128 = len(cfg.c128_layers) * abi.NATIVE_RECORD_BYTES / abi.C128_RATIO
    swa = swa_ratio * cfg.num_layers * abi.NATIVE_RECORD_BYTES
    return c4 + c128 + swa


def fixed_bytes(cfg: ModelConfig, max_requests: int) -> int:
    """Per-request state independent of context length (compressor state)."""
    comp = 0
    for r in cfg.compress_ratios:
        if r:
            comp += 3 * abi.LATENT_DIM * 4
            if r == abi.C4_RATIO:
                comp += 3 * cfg.index_dim * 4
    return max_requests * comp


def plan_capacity(cfg: ModelConfig, ecfg: EngineConfig, available_bytes: int) -> CapacityReport:
    """Token capacity for a KV budget; pages of 256 tokens."""
    bpt = bytes_per_full_token(cfg, ecfg.kv_cache_format, ecfg.swa_full_tokens_ratio, ecfg.keep_for)
    fixed = fixed_bytes(cfg, ecfg.max_running_requests)
    usable = max(0, available_bytes - fixed)
    tokens = int(usable // bpt)
    pages = tokens // (abi.RECORDS_PER_PAGE * abi.C4_RATIO)
    return CapacityReport(ecfg.kv_cache_format, bpt, available_bytes, fixed,
                          pages * abi.RECORDS_PER_PAGE * abi.C4_RATIO, pages)


class PageAllocator:
    """Free-list page allocator with reference counts (host side): a page shared by several requests
    (and the prefix-block cache) returns to the free list when its last holder releases it."""

    def __init__(self, num_pages: int):
        self.num_pages = num_pages
        self._free = list(range(num_pages - 1, -1, -1))
        self._ref = [0] * num_pages

    @property
    def free(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> list[int]:
        if n > len(self._free):
            raise MemoryError(f"KV pool exhausted: need {n} pages, {len(self._free)} free")
        pages = [self._free.pop() for _ in range(n)]
        for p in pages:
            self._ref[p] = 1
        return pages

    def share(self, pages: list[int]) -> None:
        """One more holder of each (allocated) page."""
        for p in pages:
            if self._ref[p] <= 0:
                raise ValueError(f"page {p} is not allocated")
            self._ref[p] += 1

    def refs(self, page: int) -> int:
        return self._ref[page]

    def release(self, pages: list[int]) -> None:
        for p in pages:
            if self._ref[p] <= 0:
                raise ValueError(f"page {p} released more often than held")
            self._ref[p] -= 1
            if self._ref[p] == 0:
                self._free.append(p)


class KVPool:
    """All per-rank KV storage for one model.  Tensors live on `device`."""

    TOKENS_PER_PAGE = abi.RECORDS_PER_PAGE * abi.C4_RATIO  # 256
    TOKENS_PER_C128_PAGE = abi.RECORDS_PER_PAGE * abi.C128_RATIO  # 8192

    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig, num_pages: int, max_requests: int,
                 max_context: int, device):
        ecfg.validate()
        self.cfg, self.ecfg = cfg, ecfg
        self.device = torch.device(device)
        self.kv_format = ecfg.kv_cache_format
        self.num_pages = num_pages
        self.max_requests = max_requests
        self.max_context = max_context
        self.max_pages_per_req = (max_context + self.TOKENS_PER_PAGE - 1) // self.TOKENS_PER_PAGE
        self.max_c128_pages_per_req = (max_context + self.TOKENS_PER_C128_PAGE - 1) // self.TOKENS_PER_C128_PAGE
        # C128 pages are budgeted from the C4 pages (1 C128 page per 32 C4 pages) + 1 per request
        self.num_c128_pages = num_pages // 32 + max_requests
        dev = self.device
        rows = num_pages * abi.RECORDS_PER_PAGE
        self.c4_native: dict[int, torch.Tensor] = {}
        self.c4_values: dict[int, torch.Tensor] = {}
        self.c4_bitmap: dict[int, torch.Tensor] = {}
        self.c4_scales: dict[int, torch.Tensor] = {}
        self.c4_fp4: dict[int, torch.Tensor] = {}
        # FP4 formats: "native" / "direct" (pages of packmla.formats.fp4), None for the FP8 formats
        self.fp4_format = self.kv_format[4:] if self.kv_format.startswith("fp4-") else None
        self.index_keys: dict[int, torch.Tensor] = {}
        self.index_scales: dict[int, torch.Tensor] = {}
        unknown = set(ecfg.layer_keep_counts or {}) - set(cfg.c4_layers)
        if unknown:
            raise ValueError(f"survivor counts for layers without C4 records: {sorted(unknown)}")
        self.keep = {layer: ecfg.keep_for(layer) for layer in cfg.c4_layers}
        for layer in cfg.c4_layers:
            if self.fp4_format is not None:
                self.c4_fp4[layer] = torch.zeros(num_pages * fp4.page_bytes(self.fp4_format), dtype=torch.uint8,
                                                 device=dev)
            elif self.kv_format == "direct":
                self.c4_values[layer] = torch.zeros(rows, self.keep[layer], dtype=torch.uint8, device=dev)
                self.c4_bitmap[layer] = torch.zeros(rows, abi.BITMAP_WORDS, dtype=torch.int64, device=dev)
                self.c4_scales[layer] = torch.zeros(rows, abi.NUM_TILES, dtype=torch.uint8, device=dev)
            else:
                self.c4_native[layer] = torch.zeros(num_pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
            # one extra trailing "trash" row absorbs writes of rows without a destination
            self.index_keys[layer] = torch.zeros(rows + 1, cfg.index_dim, dtype=torch.uint8, device=dev)
            self.index_scales[layer] = torch.zeros(rows + 1, dtype=torch.float32, device=dev)
        self.c128_native = {
            layer: torch.zeros(self.num_c128_pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
            for layer in cfg.c128_layers
        }
        swa_pages = max_requests * cfg.window // abi.RECORDS_PER_PAGE
        self.swa = [torch.zeros(swa_pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
                    for _ in range(cfg.num_layers)]
        # compressor pooling state: [max_requests, 3, dim] = (running max, sum of exp, weighted sum)
        self.comp_state: dict[int, torch.Tensor] = {}
        self.index_state: dict[int, torch.Tensor] = {}
        for layer, r in enumerate(cfg.compress_ratios):
            if r:
                self.comp_state[layer] = self._fresh_state(max_requests, abi.LATENT_DIM)
                if r == abi.C4_RATIO:
                    self.index_state[layer] = self._fresh_state(max_requests, cfg.index_dim)
        self.page_table = torch.full((max_requests, self.max_pages_per_req), -1, dtype=torch.int32, device=dev)
        self.c128_table = torch.full((max_requests, self.max_c128_pages_per_req), -1, dtype=torch.int32, device=dev)
        self.pages = PageAllocator(num_pages)
        self.c128_pages = PageAllocator(self.num_c128_pages)
        self._req_pages: dict[int, list[int]] = {}
        self._req_c128: dict[int, list[int]] = {}
        self._free_slots = list(range(max_requests - 1, -1, -1))

    def _fresh_state(self, n: int, dim: int) -> torch.Tensor:
        st = torch.zeros(n, 3, dim, dtype=torch.float32, device=self.device)
        st[:, 0] = float("-inf")
        return st

    # ------------------------------------------------------------------ bytes
    def device_bytes(self) -> int:
        total = 0
        for d in (self.c4_native, self.c4_values, self.c4_bitmap, self.c4_scales, self.c4_fp4, self.index_keys,
                  self.index_scales, self.c128_native, self.comp_state, self.index_state):
            total += sum(t.numel() * t.element_size() for t in d.values())
        total += sum(t.numel() * t.element_size() for t in self.swa)
        return total

    # ------------------------------------------------------------------ requests
    def admit(self, tokens: int, shared_pages: list[int] | None = None,
              shared_c128: list[int] | None = None) -> int:
        """Reserve a request slot with pages for `tokens` tokens; returns the slot.  `shared_pages` /
        `shared_c128`: the request's first pages, held by the prefix-block cache and shared read-only
        (the request takes one more reference on each)."""
        if not self._free_slots:
            raise MemoryError("no free request slot")
        slot = self._free_slots.pop()
        self._req_pages[slot] = []
        self._req_c128[slot] = []
        for alloc, pages, table, owned in ((self.pages, shared_pages, self.page_table, self._req_pages),
                                           (self.c128_pages, shared_c128, self.c128_table, self._req_c128)):
            if pages:
                alloc.share(pages)
                owned[slot].extend(pages)
                table[slot, :len(pages)] = torch.tensor(pages, dtype=torch.int32, device=self.device)
        try:
            self.ensure(slot, tokens)
        except MemoryError:
            self.release(slot)
            raise
        self.comp_state_reset(slot)
        return slot

    def ensure(self, slot: int, tokens: int) -> None:
        """Grow the request's page tables to cover `tokens` tokens."""
        if tokens > self.max_context:
            raise ValueError(f"context {tokens} exceeds max_context {self.max_context}")
        need = (tokens + self.TOKENS_PER_PAGE - 1) // self.TOKENS_PER_PAGE - len(self._req_pages[slot])
        if need > 0:
            new = self.pages.alloc(need)
            start = len(self._req_pages[slot])
            self._req_pages[slot].extend(new)
            self.page_table[slot, start:start + need] = torch.tensor(new, dtype=torch.int32, device=self.device)
        need = (tokens + self.TOKENS_PER_C128_PAGE - 1) // self.TOKENS_PER_C128_PAGE - len(self._req_c128[slot])
        if need > 0:
            new = self.c128_pages.alloc(need)
            start = len(self._req_c128[slot])
            self._req_c128[slot].extend(new)
            self.c128_table[slot, start:start + need] = torch.tensor(new, dtype=torch.int32, device=self.device)

    def release(self, slot: int) -> None:
        self.pages.release(self._req_pages.pop(slot, []))
        self.c128_pages.release(self._req_c128.pop(slot, []))
        self.page_table[slot] = -1
        self.c128_table[slot] = -1
        self._free_slots.append(slot)

    def clone_kv(self, src: int, dst: int, tokens: int) -> None:
        """Copy the KV of the first `tokens` tokens of request slot `src` into slot `dst` (pages already
        reserved for both): C4 planes and indexer keys of the covering pages, C128 records, the SWA ring
        and the compressor / indexer pooling state, so `dst` continues exactly where `src` stands."""
        R, PB = abi.RECORDS_PER_PAGE, abi.NATIVE_PAGE_BYTES
        n = (tokens + self.TOKENS_PER_PAGE - 1) // self.TOKENS_PER_PAGE
        n128 = (tokens + self.TOKENS_PER_C128_PAGE - 1) // self.TOKENS_PER_C128_PAGE
        dev = self.device
        sp = torch.tensor(self._req_pages[src][:n], dtype=torch.int64, device=dev)
        dp = torch.tensor(self._req_pages[dst][:n], dtype=torch.int64, device=dev)
        j = torch.arange(R, device=dev)
        srow, drow = (sp[:, None] * R + j).reshape(-1), (dp[:, None] * R + j).reshape(-1)
        for layer in self.cfg.c4_layers:
            if self.fp4_format is not None:
                pages = self.c4_fp4[layer].view(-1, fp4.page_bytes(self.fp4_format))
                pages[dp] = pages[sp]
            elif self.kv_format == "direct":
                for t in (self.c4_values[layer], self.c4_bitmap[layer], self.c4_scales[layer]):
                    t[drow] = t[srow]
            else:
                pages = self.c4_native[layer].view(-1, PB)
                pages[dp] = pages[sp]
            self.index_keys[layer][drow] = self.index_keys[layer][srow]
            self.index_scales[layer][drow] = self.index_scales[layer][srow]
        if n128:
            s128 = torch.tensor(self._req_c128[src][:n128], dtype=torch.int64, device=dev)
            d128 = torch.tensor(self._req_c128[dst][:n128], dtype=torch.int64, device=dev)
            for t in self.c128_native.values():
                pages = t.view(-1, PB)
                pages[d128] = pages[s128]
        slot_bytes = (self.cfg.window // R) * PB
        for t in self.swa:
            ring = t.view(-1, slot_bytes)
            ring[dst] = ring[src]
        for st in list(self.comp_state.values()) + list(self.index_state.values()):
            st[dst] = st[src]

    def comp_state_reset(self, slot: int) -> None:
        for st in list(self.comp_state.values()) + list(self.index_state.values()):
            st[slot, 0] = float("-inf")
            st[slot, 1:] = 0

    @property
    def free_tokens(self) -> int:
        return self.pages.free * self.TOKENS_PER_PAGE

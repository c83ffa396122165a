"""GLM-5.3 MLA KV pool: the persistent row planes of the eleven MLA layers, request pages and capacity.

Reference behaviour (third_party/README.md:440-465): `--kv-cache-format direct` selects the 320-byte Packed
MLA pool.  Eleven MLA layers own two persistent planes per slot (256 raw E4M3 bytes and eight uint64
bitmap words), Native keeps 512-byte rows.  The producer writes each row once.  The indexer keys stay as
they are, and startup rejects unsupported combinations before pool allocation: FP8 KV, the pinned text
geometry and a BF16 model dtype are required, and HiCache and the DeepSeek codec overrides are refused
(scripts/local/run-server.sh:94-97).

Here a pool holds, per MLA layer, the rows (Native [rows, 512] or Packed values [rows, 256] + bitmap
[rows, 8]) and the indexer keys (128 E4M3 codes + an fp32 scale per row).  Rows are handed out in pages of
64 tokens through the refcounted `PageAllocator`, and a request's token t lives in row
`page_table[slot, t // 64] * 64 + t % 64`.  Stores and decode go through `packmla.ops.glm`.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..formats import glm
from ..ops.glm import GLMPlanes, glm_sparse_decode, glm_store
from .pool import PageAllocator

TOKENS_PER_PAGE = 64


@dataclass
class GLMCacheConfig:
    kv_cache_format: str = "native"  # native | direct
    kv_cache_dtype: str = "fp8_e4m3"
    model_dtype: str = "bfloat16"
    enable_hierarchical_cache: bool = False
    keep_count: int | None = None  # DeepSeek codec overrides: not supported for GLM
    geometry: glm.GLMGeometry = glm.GLM53

    def validate(self) -> None:
        """Refuse unsupported combinations before any allocation."""
        if self.kv_cache_format not in ("native", "direct"):
            raise ValueError("GLM kv_cache_format must be native or direct")
        if self.kv_cache_dtype != "fp8_e4m3":
            raise ValueError("GLM MLA rows require the FP8 (e4m3) KV cache")
        if self.model_dtype != "bfloat16":
            raise ValueError("GLM MLA rows require a BF16 model dtype")
        if self.enable_hierarchical_cache or self.keep_count is not None:
            raise ValueError("the GLM MLA pool takes neither the host tier nor a C4 survivor-count setting")
        g = self.geometry
        if (g.kv_lora_rank, g.qk_head_dim, len(g.mla_layers)) != (glm.LATENT_DIM, 256, 11):
            raise ValueError("GLM MLA rows require the pinned GLM-5.3 text geometry")


def bytes_per_token(cfg: GLMCacheConfig) -> int:
    return glm.bytes_per_token(cfg.kv_cache_format, cfg.geometry)


def capacity_tokens(cfg: GLMCacheConfig, budget_bytes: int) -> int:
    """Whole pages of tokens that `budget_bytes` holds in this format."""
    return budget_bytes // (bytes_per_token(cfg) * TOKENS_PER_PAGE) * TOKENS_PER_PAGE


class GLMKVPool:
    def __init__(self, cfg: GLMCacheConfig, num_pages: int, max_requests: int, max_context: int, device):
        cfg.validate()
        self.cfg = cfg
        self.device = torch.device(device)
        self.num_pages = num_pages
        self.max_requests = max_requests
        self.max_context = max_context
        rows = num_pages * TOKENS_PER_PAGE
        dev = self.device
        g = cfg.geometry
        self.packed = cfg.kv_cache_format == "direct"
        self.rows: dict[int, torch.Tensor] = {}
        self.planes: dict[int, GLMPlanes] = {}
        for layer in g.mla_layers:
            if self.packed:
                self.planes[layer] = GLMPlanes(torch.zeros(rows, glm.PACKED_KEEP, dtype=torch.uint8, device=dev),
                                               torch.zeros(rows, glm.BITMAP_WORDS, dtype=torch.int64, device=dev))
            else:
                self.rows[layer] = torch.zeros(rows, glm.NATIVE_ROW_BYTES, dtype=torch.uint8, device=dev)
        self.index_keys = {l: torch.zeros(rows, g.index_head_dim, dtype=torch.uint8, device=dev) for l in g.mla_layers}
        self.index_scales = {l: torch.zeros(rows, dtype=torch.float32, device=dev) for l in g.mla_layers}
        self.pages = PageAllocator(num_pages)
        self.max_pages_per_req = -(-max_context // TOKENS_PER_PAGE)
        self.page_table = torch.full((max_requests, self.max_pages_per_req), -1, dtype=torch.int32, device=dev)
        self._req_pages: list[list[int]] = [[] for _ in range(max_requests)]
        self._free_slots = list(range(max_requests - 1, -1, -1))

    # ------------------------------------------------------------------ lifecycle
    def admit(self, tokens: int) -> int:
        if not self._free_slots:
            raise MemoryError("no free request slot")
        slot = self._free_slots.pop()
        self._req_pages[slot] = []
        try:
            self.ensure(slot, tokens)
        except MemoryError:
            self.release(slot)
            raise
        return slot

    def ensure(self, slot: int, tokens: int) -> None:
        if tokens > self.max_context:
            raise ValueError(f"context {tokens} exceeds max_context {self.max_context}")
        need = -(-tokens // TOKENS_PER_PAGE) - len(self._req_pages[slot])
        if need > 0:
            new = self.pages.alloc(need)
            start = len(self._req_pages[slot])
            self._req_pages[slot].extend(new)
            self.page_table[slot, start:start + need] = torch.tensor(new, dtype=torch.int32, device=self.device)

    def release(self, slot: int) -> None:
        self.pages.release(self._req_pages[slot])
        self._req_pages[slot] = []
        self.page_table[slot] = -1
        self._free_slots.append(slot)

    def rows_of(self, slot: int, positions: torch.Tensor) -> torch.Tensor:
        """Physical rows of token positions of request `slot` (int64, -1 for positions past its pages)."""
        pos = positions.to(self.device, torch.int64)
        idx = pos // TOKENS_PER_PAGE
        inside = (pos >= 0) & (idx < self.max_pages_per_req)
        page = self.page_table[slot].to(torch.int64)[idx.clamp(0, self.max_pages_per_req - 1)]
        return torch.where(inside & (page >= 0), page * TOKENS_PER_PAGE + pos % TOKENS_PER_PAGE,
                           torch.full_like(pos, -1))

    # ------------------------------------------------------------------ data path
    def store(self, layer: int, raw: torch.Tensor, weight: torch.Tensor, eps: float, slot: int,
              positions: torch.Tensor) -> None:
        """Write the latent rows (before the norm) of `positions` of request `slot` for MLA `layer`."""
        rows = self.rows_of(slot, positions)
        if self.packed:
            glm_store(raw, weight, eps, rows, planes=self.planes[layer])
        else:
            glm_store(raw, weight, eps, rows, pool=self.rows[layer])

    def decode(self, layer: int, q: torch.Tensor, rows: torch.Tensor, lens: torch.Tensor, **kw):
        """Sparse decode of `layer` over physical `rows` int32 [B, K] (first `lens[b]` used)."""
        if self.packed:
            return glm_sparse_decode(q, rows, lens, planes=self.planes[layer], **kw)
        return glm_sparse_decode(q, rows, lens, pool=self.rows[layer], **kw)

    def device_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   list(self.rows.values()) + [p.values for p in self.planes.values()] +
                   [p.bitmap for p in self.planes.values()] + list(self.index_keys.values()) +
                   list(self.index_scales.values()))

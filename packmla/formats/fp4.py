"""FP4 C4 record codec (the V4.1 cache extension): Native 288 B and Packed 224 B records, CPU oracle.

Format (reference: third_party/README.md:120-141, the software codec `fp4_cache.py` of its V4.1 fork):

Native FP4 record, 288 logical bytes
    codes   256 B   512 E2M1 codes, two per byte, coordinate 2i in the low nibble of byte i
    scales   32 B   one E4M3 scale per 16 consecutive coordinates
Packed FP4 record, 224 logical bytes (the 256 largest dequantized magnitudes of the Native record)
    codes   128 B   the 256 survivors' codes in ascending coordinate order, even ranks in low nibbles
    bitmap   64 B   8 uint64 words, MSB-first: coordinate 64 w + b is bit 63 - b of word w
    scales   32 B   unchanged (looked up by the survivor's original 16-coordinate group)

Rows enter already normalized, rotated (RoPE applied to the tail) and rounded to BF16: FP4 records
hold rotated values, unlike the FP8 Packed records.  Survivor selection happens after quantization,
on the dequantized magnitudes, and ties keep the lower coordinate, so codes and scales of survivors
are those of the Native record.  Pages keep all data rows, then all scale rows.

The quantization rounding is packmla's definition (the reference's notes state the scale grain, not
the rounding): scale = E4M3(amax / 6) with round-to-nearest-even (the largest E2M1 magnitude is 6),
code = E2M1(x / scale) with round-to-nearest, ties to the even code, saturating at 6.
"""
from __future__ import annotations

import torch

from . import abi, codec

GROUP = 16
GROUPS = abi.LATENT_DIM // GROUP          # 32 scale bytes
KEEP = abi.PACKED_KEEP                    # 256 survivors
NATIVE_CODE_BYTES = abi.LATENT_DIM // 2   # 256
PACKED_CODE_BYTES = KEEP // 2             # 128
BITMAP_BYTES = abi.LATENT_DIM // 8        # 64
NATIVE_RECORD_BYTES = NATIVE_CODE_BYTES + GROUPS            # 288
PACKED_RECORD_BYTES = PACKED_CODE_BYTES + BITMAP_BYTES + GROUPS  # 224

# E2M1 magnitudes by 3-bit code (bit 3 of a nibble is the sign)
E2M1_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_encode(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> 4-bit codes (uint8 0..15): nearest grid magnitude, ties to the even code, saturating."""
    a = x.abs().clamp(max=6.0)
    grid = E2M1_GRID.to(x.device)
    d = (a[..., None] - grid).abs()
    best = d.min(-1, keepdim=True).values
    tied = d == best
    # among equally near grid points prefer the even code (the one with a zero mantissa bit)
    codes = torch.arange(8, device=x.device)
    pref = torch.where(tied, (codes % 2) * 8 + codes, torch.full_like(codes, 1 << 10))
    mag = pref.argmin(-1).to(torch.uint8)
    sign = ((x < 0) & (mag > 0)).to(torch.uint8) << 3
    return mag | sign


def e2m1_decode(codes: torch.Tensor) -> torch.Tensor:
    grid = E2M1_GRID.to(codes.device)
    v = grid[(codes & 7).long()]
    return torch.where((codes & 8) > 0, -v, v)


def _scales(rows: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-16 E4M3 scale codes (uint8) and their fp32 values."""
    amax = rows.view(rows.shape[0], GROUPS, GROUP).abs().amax(-1)
    s = (amax / 6.0).clamp(max=448.0).to(torch.float8_e4m3fn)  # E4M3 has no infinity: saturate
    return s.view(torch.uint8), s.float()


def native_encode(rows: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotated BF16-valued rows [R, 512] -> (codes uint8 [R, 256], scales uint8 [R, 32])."""
    rows = rows.float()
    s_codes, s = _scales(rows)
    q = rows.view(rows.shape[0], GROUPS, GROUP) / torch.where(s > 0, s, torch.ones_like(s))[..., None]
    c = e2m1_encode(q).view(rows.shape[0], abi.LATENT_DIM)
    c = torch.where((s > 0).repeat_interleave(GROUP, -1), c, torch.zeros_like(c))
    return (c[:, 0::2] | (c[:, 1::2] << 4)).contiguous(), s_codes.contiguous()


def _unpack_nibbles(b: torch.Tensor) -> torch.Tensor:
    return torch.stack((b & 0xF, b >> 4), -1).reshape(b.shape[0], -1)


def native_decode(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Native FP4 planes -> fp32 rows [R, 512] (BF16-valued)."""
    v = e2m1_decode(_unpack_nibbles(codes)).view(codes.shape[0], GROUPS, GROUP)
    s = scales.view(torch.float8_e4m3fn).float()
    return (v * s[..., None]).view(codes.shape[0], abi.LATENT_DIM).to(torch.bfloat16).float()


def survivor_mask(codes: torch.Tensor, scales: torch.Tensor, keep: int = KEEP) -> torch.Tensor:
    """The `keep` largest dequantized magnitudes of each Native record; ties keep the lower coordinate."""
    mag = native_decode(codes, scales).abs()
    order = torch.sort(mag, dim=-1, descending=True, stable=True).indices
    mask = torch.zeros_like(mag, dtype=torch.bool)
    mask.scatter_(-1, order[:, :keep], True)
    return mask


def bitmap_msb_first(mask: torch.Tensor) -> torch.Tensor:
    """bool [R, 512] -> int64 [R, 8], coordinate 64 w + b at bit 63 - b of word w (two's complement)."""
    bits = mask.view(mask.shape[0], 8, 64).to(torch.int64)
    weights = torch.ones(64, dtype=torch.int64, device=mask.device) << (63 - torch.arange(64, device=mask.device))
    return (bits * weights).sum(-1)


def mask_from_msb_bitmap(words: torch.Tensor) -> torch.Tensor:
    shifts = 63 - torch.arange(64, dtype=torch.int64, device=words.device)
    return ((words.to(torch.int64)[..., None] >> shifts) & 1).reshape(words.shape[0], abi.LATENT_DIM).bool()


def packed_encode(rows: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rows [R, 512] -> (survivor codes uint8 [R, 128], MSB-first bitmap int64 [R, 8], scales uint8 [R, 32])."""
    codes, scales = native_encode(rows)
    mask = survivor_mask(codes, scales)
    nib = _unpack_nibbles(codes)[mask].view(rows.shape[0], KEEP)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).contiguous()
    return packed, bitmap_msb_first(mask), scales


def packed_decode(codes: torch.Tensor, bitmap: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Packed FP4 planes -> fp32 rows [R, 512] (BF16-valued, pruned coordinates zero)."""
    R = codes.shape[0]
    mask = mask_from_msb_bitmap(bitmap)
    nib = torch.zeros(R, abi.LATENT_DIM, dtype=torch.uint8, device=codes.device)
    nib[mask] = _unpack_nibbles(codes).reshape(-1)
    full = (nib[:, 0::2] | (nib[:, 1::2] << 4))
    return native_decode(full, scales) * mask


def record_bytes(kv_format: str) -> int:
    return PACKED_RECORD_BYTES if kv_format == "direct" else NATIVE_RECORD_BYTES


def rotated_rows(normalized: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Normalized BF16-valued rows [R, 512] -> RoPE applied to the 64-coordinate tail, rounded to BF16:
    the values an FP4 record stores."""
    y = codec.rotate_tail(normalized.float().to(torch.bfloat16).float(), freqs)
    return y.to(torch.bfloat16).float()


# --------------------------------------------------------------------------- pages
def page_bytes(kv_format: str, records: int = abi.RECORDS_PER_PAGE) -> int:
    return records * record_bytes(kv_format)


def write_page(kv_format: str, rows: torch.Tensor) -> torch.Tensor:
    """Rotated rows [P, 512] -> one page uint8 [P * record bytes]: all data rows, then all scale rows.

    Native data row = 256 code bytes; Packed data row = 128 survivor code bytes + 8 MSB-first
    bitmap words (little-endian bytes).  Scale rows are the 32 E4M3 bytes of each record."""
    if kv_format == "direct":
        codes, words, scales = packed_encode(rows)
        data = torch.cat((codes, words.contiguous().view(torch.uint8).view(rows.shape[0], BITMAP_BYTES)), -1)
    else:
        data, scales = native_encode(rows)
    return torch.cat((data.reshape(-1), scales.reshape(-1)))


def read_page(kv_format: str, page: torch.Tensor, records: int = abi.RECORDS_PER_PAGE) -> torch.Tensor:
    """One page -> fp32 rows [records, 512] (Packed: pruned coordinates zero)."""
    data_row = record_bytes(kv_format) - GROUPS
    data = page[: records * data_row].view(records, data_row)
    scales = page[records * data_row: records * (data_row + GROUPS)].view(records, GROUPS)
    if kv_format == "direct":
        words = data[:, PACKED_CODE_BYTES:].contiguous().view(torch.int64)
        return packed_decode(data[:, :PACKED_CODE_BYTES].contiguous(), words, scales.contiguous())
    return native_decode(data.contiguous(), scales.contiguous())


# --------------------------------------------------------------------------- Direct decode (reference)
def gather_rows(pool: torch.Tensor, kv_format: str, indices: torch.Tensor,
                records: int = abi.RECORDS_PER_PAGE) -> torch.Tensor:
    """Paged FP4 pool uint8 [num_pages, page bytes] and record ids [N] -> rotated rows fp32 [N, 512]
    (record id = page * records + row; ids < 0 give zero rows).  Only the named records are decoded."""
    ids = indices.reshape(-1).long()
    out = torch.zeros(ids.numel(), abi.LATENT_DIM)
    valid = ids >= 0
    if not bool(valid.any()):
        return out
    pool = pool.reshape(-1, page_bytes(kv_format, records))
    data_row = record_bytes(kv_format) - GROUPS
    page, row = ids[valid] // records, ids[valid] % records
    data_off = row[:, None] * data_row + torch.arange(data_row)
    scale_off = records * data_row + row[:, None] * GROUPS + torch.arange(GROUPS)
    data = pool[page[:, None], data_off]
    scales = pool[page[:, None], scale_off]
    if kv_format == "direct":
        words = data[:, PACKED_CODE_BYTES:].contiguous().view(torch.int64)
        out[valid] = packed_decode(data[:, :PACKED_CODE_BYTES].contiguous(), words, scales)
    else:
        out[valid] = native_decode(data.contiguous(), scales)
    return out


def sparse_decode_reference(q: torch.Tensor, pool: torch.Tensor, kv_format: str, indices: torch.Tensor,
                            lens: torch.Tensor, swa_rows: list[torch.Tensor], sink: torch.Tensor, scale: float,
                            q_freqs: torch.Tensor):
    """fp32 reference of sparse MLA decode over FP4 global records beside BF16 SWA rows (the V4.1 FP4
    Native / Direct read, reference: third_party/README.md:135-141): query b attends to its SWA rows and
    to the first lens[b] selected records that are not -1 (records hold RoPE-rotated values, so no
    rotation happens at read).  Returns (out bf16 [B, H, 512], lse [B, H])."""
    from ..oracle.attention import sparse_mla_decode

    rows = []
    for b in range(q.shape[0]):
        sel = indices[b, : int(lens[b])]
        sel = sel[sel >= 0]
        rows.append(torch.cat((swa_rows[b].float(), gather_rows(pool, kv_format, sel))))
    return sparse_mla_decode(q, rows, sink, scale, q_freqs)


# --------------------------------------------------------------------------- capacity
def capacity_tokens(model_cfg, kv_format: str, budget_bytes: int, swa_ratio: float = 0.1) -> int:
    """KV token capacity of `budget_bytes` with FP4 C4 records (Native 288 B or Packed 224 B) and
    everything else as the FP8 pool accounts it (indexer keys, C128 records, SWA share)."""
    from ..kv.pool import bytes_per_full_token

    fp8 = bytes_per_full_token(model_cfg, "native", swa_ratio)
    c4_layers = len(model_cfg.c4_layers)
    bpt = fp8 + c4_layers * (record_bytes(kv_format) - abi.NATIVE_RECORD_BYTES) / abi.C4_RATIO
    return int(budget_bytes // bpt)

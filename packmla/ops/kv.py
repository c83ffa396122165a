"""KV store ops: FP32 compressor rows -> Native pages or Packed planes.

CUDA tensors run the sm_100a store kernels (csrc/kv_store.cu); CPU tensors run the
oracle codec (packmla/formats/codec.py).  Both write the same bytes.
"""
from __future__ import annotations

import torch

from ..formats import abi, codec
from ._ext import error_word, ext


def freq_table_f32(freqs_complex: torch.Tensor) -> torch.Tensor:
    """complex64 [P, 32] -> float32 [P, 32, 2] (cos, sin) contiguous."""
    return torch.view_as_real(freqs_complex.to(torch.complex64)).contiguous()


def native_store(
    raw: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    slots: torch.Tensor,
    positions: torch.Tensor,
    freqs: torch.Tensor,
    pool: torch.Tensor,
) -> None:
    """Write Native records for rows `raw` [R,512] at physical `slots` (-1 = skip).

    `positions` are the RoPE table rows (token positions); `freqs` is float32 [P,32,2];
    `pool` is uint8 pages of 64 records (data rows then scale rows).
    """
    if raw.is_cuda:
        ext().native_store(raw, weight, float(eps), slots.to(torch.int64), positions.to(torch.int64), freqs, pool,
                           error_word(raw.device))
        return
    keep = slots >= 0
    if not bool(keep.any()):
        return
    fr = torch.view_as_complex(freqs[positions[keep].long()].contiguous())
    rec = codec.native_encode(raw[keep].float(), weight.float(), eps, fr)
    pages = pool.view(-1, abi.NATIVE_PAGE_BYTES)
    for s, row in zip(slots[keep].tolist(), rec):
        page, r = divmod(s, abi.RECORDS_PER_PAGE)
        pages[page, r * abi.NATIVE_DATA_BYTES : (r + 1) * abi.NATIVE_DATA_BYTES] = row[: abi.NATIVE_DATA_BYTES]
        off = abi.RECORDS_PER_PAGE * abi.NATIVE_DATA_BYTES + r * abi.NATIVE_SCALE_BYTES
        pages[page, off : off + abi.NATIVE_SCALE_BYTES] = row[abi.NATIVE_DATA_BYTES :]


def packed_store(
    raw: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    slots: torch.Tensor,
    values: torch.Tensor,
    bitmap: torch.Tensor,
    scales: torch.Tensor,
) -> None:
    """Select the top-K |raw| (K = values.shape[1]: 256 by default, 64 .. 448 in steps of 64 for per-layer
    layouts), masked RMSNorm, quantize and write the three planes at `slots`."""
    if raw.is_cuda:
        ext().packed_store(raw, weight, float(eps), slots.to(torch.int64), values, bitmap, scales,
                           error_word(raw.device))
        return
    keep = slots >= 0
    if not bool(keep.any()):
        return
    v, b, s = codec.packed_encode(raw[keep].float(), weight.float(), eps, keep=values.shape[1])
    idx = slots[keep].long()
    values[idx] = v
    bitmap[idx] = b
    scales[idx] = s


def native_pool_read(pool: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
    """Gather Native records [R, 584] (logical order) from a paged pool (CPU or CUDA)."""
    pages = pool.view(-1, abi.NATIVE_PAGE_BYTES)
    s = slots.long()
    page, r = s // abi.RECORDS_PER_PAGE, s % abi.RECORDS_PER_PAGE
    d_idx = r[:, None] * abi.NATIVE_DATA_BYTES + torch.arange(abi.NATIVE_DATA_BYTES, device=pool.device)[None]
    s_idx = (abi.RECORDS_PER_PAGE * abi.NATIVE_DATA_BYTES + r[:, None] * abi.NATIVE_SCALE_BYTES
             + torch.arange(abi.NATIVE_SCALE_BYTES, device=pool.device)[None])
    data = pages[page[:, None], d_idx]
    sc = pages[page[:, None], s_idx]
    return torch.cat((data, sc), -1)


def packed_to_native(values: torch.Tensor, bitmap: torch.Tensor, scales: torch.Tensor, rows: torch.Tensor,
                     positions: torch.Tensor, freqs: torch.Tensor, out: torch.Tensor, dst: torch.Tensor) -> None:
    """Adapter: write the Native record of Packed row `rows[i]` (RoPE at `positions[i]`) at slot `dst[i]`
    of the Native pages `out` (dst -1 = skip).  `freqs` is float32 [P, 32, 2]."""
    if values.is_cuda:
        ext().packed_to_native(values, bitmap, scales, rows.to(torch.int32).contiguous(),
                               positions.to(torch.int32).contiguous(), freqs, out, dst.to(torch.int64).contiguous(),
                               error_word(values.device))
        return
    keep = dst >= 0
    r, p, d = rows[keep].long(), positions[keep].long(), dst[keep].long()
    fr = torch.complex(freqs[p, :, 0], freqs[p, :, 1])
    recs = codec.native_from_packed(values[r], bitmap[r], scales[r], fr)
    pages = out.view(-1, abi.NATIVE_PAGE_BYTES)
    page, rr = d // abi.RECORDS_PER_PAGE, d % abi.RECORDS_PER_PAGE
    for i in range(recs.shape[0]):
        base_d = int(rr[i]) * abi.NATIVE_DATA_BYTES
        base_s = abi.RECORDS_PER_PAGE * abi.NATIVE_DATA_BYTES + int(rr[i]) * abi.NATIVE_SCALE_BYTES
        pages[page[i], base_d:base_d + abi.NATIVE_DATA_BYTES] = recs[i, :abi.NATIVE_DATA_BYTES]
        pages[page[i], base_s:base_s + abi.NATIVE_SCALE_BYTES] = recs[i, abi.NATIVE_DATA_BYTES:]


def fp4_store(raw: torch.Tensor, weight: torch.Tensor, eps: float, slots: torch.Tensor, positions: torch.Tensor,
              freqs: torch.Tensor, pool: torch.Tensor, packed: bool) -> None:
    """Write FP4 C4 records (the V4.1 cache, packmla/formats/fp4.py) for rows `raw` [R, 512] at physical
    `slots` (-1 = skip): Native 288 B or, with `packed`, Packed 224 B, in pages of 64 records (data rows, then
    scale rows).  `positions` are the RoPE rows; the records hold the normalized, tail-rotated values."""
    from ..formats import fp4

    if raw.is_cuda:
        ext().fp4_store(raw.float().contiguous(), weight.float().contiguous(), float(eps), slots.to(torch.int64),
                        positions.to(torch.int64), freqs, pool, bool(packed), error_word(raw.device))
        return
    keep = slots >= 0
    if not bool(keep.any()):
        return
    fr = torch.view_as_complex(freqs[positions[keep].long()].contiguous())
    rows = fp4.rotated_rows(codec.rms_normalize(raw[keep].float(), weight.float(), eps), fr)
    fmt = "direct" if packed else "native"
    data_row = fp4.record_bytes(fmt) - fp4.GROUPS
    if packed:
        codes, words, scales = fp4.packed_encode(rows)
        data = torch.cat((codes, words.contiguous().view(torch.uint8).view(rows.shape[0], fp4.BITMAP_BYTES)), -1)
    else:
        data, scales = fp4.native_encode(rows)
    pages = pool.view(-1, fp4.page_bytes(fmt))
    for s, d, sc in zip(slots[keep].tolist(), data, scales):
        page, r = divmod(s, abi.RECORDS_PER_PAGE)
        pages[page, r * data_row:(r + 1) * data_row] = d
        off = abi.RECORDS_PER_PAGE * data_row + r * fp4.GROUPS
        pages[page, off:off + fp4.GROUPS] = sc


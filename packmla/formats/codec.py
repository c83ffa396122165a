"""CPU oracle codec for Native (584 B) and Packed (328 B) C4 records.

Pure PyTorch, fp32. Every CUDA store/read kernel in packmla is tested byte-exact
against these functions, so the arithmetic order here is the contract:

* RMSNorm sum of squares follows the warp layout of the store kernels: lane l of a
  32-lane warp owns coordinates {128 j + 4 l + i : j, i in 0..3}, accumulates
  x*x (rounded) into an fp32 partial in (j, i) order, then the 32 partials are
  combined by a butterfly (xor 16, 8, 4, 2, 1).  r = 1 / sqrt(sum/512 + eps) with
  IEEE division and square root, and y = bf16((x * r) * w).
* UE8M0 scale of a 64-coordinate tile: the smallest e with 448 * 2^e >= max(amax, 1e-4);
  code = e + 127.  (Same as 2^ceil(log2(max(amax,1e-4)/448)) of the reference,
  training/losses.py:90-94, training/tests/test_integration.py:1595-1605.)
* E4M3 = round-to-nearest-even of y / 2^e.
* Packed selection keeps the 256 largest |raw| (fp32, before the norm), ties to the
  lower coordinate; the norm is the masked RMSNorm (mean over all 512 coordinates).
* Reads dequantize, zero-fill pruned coordinates, round to BF16, then rotate the
  tail as 32 adjacent complex pairs (2i, 2i+1): re' = re*c - im*s, im' = re*s + im*c,
  and round to BF16 again (candidate-sglang.patch `_unpack_gather_bf16_rope_kernel`).
"""

from __future__ import annotations

import torch

from . import abi

_F32 = torch.float32
_BF16 = torch.bfloat16


# --------------------------------------------------------------------------- scalars
def ue8m0_exponent(amax: torch.Tensor) -> torch.Tensor:
    """Exact smallest e with 448 * 2^e >= max(amax, 1e-4) (amax fp32, non-negative)."""
    a = amax.to(_F32).clamp_min(abi.AMAX_FLOOR)  # the Python float becomes an fp32 scalar on amax's device
    mant, exp = torch.frexp(a)  # a = mant * 2^exp, mant in [0.5, 1)
    return (exp - 9 + (mant > 0.875).to(exp.dtype)).to(torch.int32)


def e4m3_encode(v: torch.Tensor) -> torch.Tensor:
    return v.to(_F32).to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_decode(codes: torch.Tensor) -> torch.Tensor:
    return codes.view(torch.float8_e4m3fn).to(_F32)


def exp2_int(e: torch.Tensor) -> torch.Tensor:
    return torch.ldexp(torch.ones_like(e, dtype=_F32), e.to(torch.int32))


# --------------------------------------------------------------------------- norm
def _lane_order_sumsq(x: torch.Tensor) -> torch.Tensor:
    """Sum of squares of [R, 512] fp32 rows in the store kernels' warp order."""
    r = x.shape[0]
    sq = (x * x).to(_F32)  # each square rounded to fp32
    # coordinate 128 j + 4 l + i -> [R, j, l, i]
    lanes = sq.view(r, 4, 32, 4)
    acc = torch.zeros(r, 32, dtype=_F32, device=x.device)
    for j in range(4):
        for i in range(4):
            acc = acc + lanes[:, j, :, i]
    idx = torch.arange(32, device=x.device)
    for off in (16, 8, 4, 2, 1):
        acc = acc + acc[:, idx ^ off]
    return acc[:, 0]


def rms_normalize(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """bf16((x * r) * w) with r = 1/sqrt(mean(x^2) + eps); returns fp32 holding bf16 values."""
    x = x.to(_F32)
    ss = _lane_order_sumsq(x)
    r = 1.0 / torch.sqrt(ss / abi.LATENT_DIM + torch.tensor(eps, dtype=_F32))
    y = (x * r[:, None]) * weight.to(_F32)[None, :]
    return y.to(_BF16).to(_F32)


# --------------------------------------------------------------------------- rope
def rope_table(max_positions: int, theta: float = 10000.0, dim: int = abi.ROPE_DIM) -> torch.Tensor:
    """complex64 [max_positions, dim/2]: exp(i * pos * theta^(-2k/dim))."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    ang = torch.outer(torch.arange(max_positions, dtype=torch.float64), inv)
    return torch.polar(torch.ones_like(ang), ang).to(torch.complex64)


def rotate_tail(x: torch.Tensor, freqs: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """Rotate coordinates 448..511 of fp32 rows [..., 512] by complex freqs [..., 32]."""
    out = x.to(_F32).clone()
    tail = out[..., abi.NOPE_DIM :].reshape(*out.shape[:-1], abi.ROPE_PAIRS, 2)
    fr = torch.view_as_real(freqs.to(torch.complex64)).to(_F32)
    c, s = fr[..., 0], fr[..., 1]
    if inverse:
        s = -s
    re, im = tail[..., 0], tail[..., 1]
    new_re = re * c - im * s
    new_im = re * s + im * c
    out[..., abi.NOPE_DIM :] = torch.stack((new_re, new_im), -1).reshape(*out.shape[:-1], abi.ROPE_DIM)
    return out


# --------------------------------------------------------------------------- tiles
def quantize_tiles(y: torch.Tensor, ntiles: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize fp32 (bf16-valued) [R, 64*ntiles] into (e4m3 codes uint8, ue8m0 codes uint8 [R, ntiles])."""
    r = y.shape[0]
    t = y[:, : ntiles * abi.TILE].reshape(r, ntiles, abi.TILE)
    amax = t.abs().amax(-1)
    e = ue8m0_exponent(amax)
    q = e4m3_encode(t * exp2_int(-e)[..., None]).reshape(r, ntiles * abi.TILE)
    return q, (e + abi.UE8M0_BIAS).to(torch.uint8)


def dequant_tiles(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    r, n = codes.shape
    ntiles = n // abi.TILE
    s = exp2_int(scales[:, :ntiles].to(torch.int32) - abi.UE8M0_BIAS)
    return (e4m3_decode(codes).reshape(r, ntiles, abi.TILE) * s[..., None]).reshape(r, n)


# --------------------------------------------------------------------------- native
def native_encode(raw: torch.Tensor, weight: torch.Tensor, eps: float, freqs: torch.Tensor) -> torch.Tensor:
    """FP32 compressor rows [R,512] -> Native records uint8 [R, 584] (logical order)."""
    return _native_pack(rms_normalize(raw, weight, eps), freqs)


def native_from_packed(values, bitmap, scales, freqs) -> torch.Tensor:
    """Adapter view of Packed records: the Native record of the decoded (pruned) row.

    NoPE tiles are re-quantized from the exactly decoded values (UE8M0 of the tile's amax); the tail
    is rotated by `freqs` [R, 32] and rounded to BF16.
    """
    return _native_pack(packed_decode(values, bitmap, scales), freqs)


def _native_pack(y: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """bf16-valued rows [R, 512] -> Native records [R, 584]."""
    q, sc = quantize_tiles(y[:, : abi.NOPE_DIM], abi.NOPE_TILES)
    tail = rotate_tail(y, freqs)[:, abi.NOPE_DIM :].to(_BF16)
    out = torch.zeros(y.shape[0], abi.NATIVE_RECORD_BYTES, dtype=torch.uint8, device=y.device)
    out[:, : abi.NOPE_DIM] = q
    out[:, abi.NOPE_DIM : abi.NATIVE_DATA_BYTES] = tail.contiguous().view(torch.uint8)
    out[:, abi.NATIVE_DATA_BYTES : abi.NATIVE_DATA_BYTES + abi.NOPE_TILES] = sc
    return out


def native_decode(records: torch.Tensor) -> torch.Tensor:
    """Native records [R, 584] -> fp32 [R, 512] holding bf16 values (tail already rotated)."""
    r = records.shape[0]
    nope = dequant_tiles(records[:, : abi.NOPE_DIM].contiguous(),
                         records[:, abi.NATIVE_DATA_BYTES : abi.NATIVE_DATA_BYTES + abi.NOPE_TILES].contiguous())
    tail = records[:, abi.NOPE_DIM : abi.NATIVE_DATA_BYTES].contiguous().view(_BF16).to(_F32)
    return torch.cat((nope.to(_BF16).to(_F32), tail.reshape(r, abi.ROPE_DIM)), -1)


# --------------------------------------------------------------------------- packed
def topmag_mask(raw: torch.Tensor, keep: int = abi.PACKED_KEEP) -> torch.Tensor:
    """Keep the `keep` largest |raw| per row; ties keep the lower coordinate."""
    order = torch.sort(raw.to(_F32).abs(), dim=-1, descending=True, stable=True).indices
    mask = torch.zeros_like(raw, dtype=torch.bool)
    mask.scatter_(-1, order[..., :keep], True)
    return mask


def bitmap_from_mask(mask: torch.Tensor) -> torch.Tensor:
    """bool [R, 512] -> int64 [R, 8] words (LSB-first), bit pattern identical to uint64."""
    bits = mask.view(mask.shape[0], abi.BITMAP_WORDS, 64).to(torch.int64)
    weights = torch.ones(64, dtype=torch.int64, device=mask.device) << torch.arange(64, dtype=torch.int64,
                                                                                    device=mask.device)
    return (bits * weights).sum(-1)  # wraps to the two's-complement bit pattern


def mask_from_bitmap(words: torch.Tensor) -> torch.Tensor:
    w = words.to(torch.int64)
    shifts = torch.arange(64, dtype=torch.int64, device=words.device)
    bits = (w[..., None] >> shifts) & 1
    return bits.reshape(w.shape[0], abi.LATENT_DIM).bool()


def packed_encode(
    raw: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    mask: torch.Tensor | None = None,
    keep: int = abi.PACKED_KEEP,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """FP32 rows [R,512] -> (values uint8 [R,keep], bitmap int64 [R,8], scales uint8 [R,8])."""
    raw = raw.to(_F32)
    if mask is None:
        mask = topmag_mask(raw, keep)
    if not bool((mask.sum(-1) == keep).all()):
        raise ValueError(f"mask must keep exactly {keep} coordinates per row")
    masked = raw.masked_fill(~mask, 0.0)
    y = rms_normalize(masked, weight, eps)
    codes, scales = quantize_tiles(y, abi.NUM_TILES)
    values = codes[mask].view(raw.shape[0], keep)  # row-major boolean select keeps ascending order
    return values.contiguous(), bitmap_from_mask(mask), scales.contiguous()


def packed_decode(values: torch.Tensor, bitmap: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Planes -> fp32 [R, 512] bf16-valued, pre-RoPE, pruned coordinates zero."""
    r = values.shape[0]
    mask = mask_from_bitmap(bitmap)
    codes = torch.zeros(r, abi.LATENT_DIM, dtype=torch.uint8, device=values.device)
    codes[mask] = values.reshape(-1)
    dense = dequant_tiles(codes, scales).masked_fill(~mask, 0.0)
    return dense.to(_BF16).to(_F32)


def packed_read(values, bitmap, scales, freqs) -> torch.Tensor:
    """Full read path: dequant, zero-fill, BF16 round, tail RoPE, BF16 round."""
    return rotate_tail(packed_decode(values, bitmap, scales), freqs).to(_BF16).to(_F32)


def simulated_packed_rows(raw, mask, weight, eps, freqs) -> torch.Tensor:
    """Dense simulation of any retention budget (64..448): same rounding as the 256 codec."""
    masked = raw.to(_F32).masked_fill(~mask, 0.0)
    y = rms_normalize(masked, weight, eps)
    codes, scales = quantize_tiles(y, abi.NUM_TILES)
    dense = dequant_tiles(codes, scales).masked_fill(~mask, 0.0).to(_BF16).to(_F32)
    return rotate_tail(dense, freqs).to(_BF16).to(_F32)


def native_rows(raw, weight, eps, freqs) -> torch.Tensor:
    """Decoded Native rows straight from raw (encode then decode)."""
    return native_decode(native_encode(raw, weight, eps, freqs))

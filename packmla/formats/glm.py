"""GLM-5.3-Flash MLA rows: Native (512 B) and Packed (320 B), CPU oracle.

Reference behaviour (third_party/README.md:440-465, the GLM-5.3-Flash candidate): eleven MLA layers
(the `deepseek_sparse_attention` layers 3, 7, ..., 43 of the 45; the others are KDA linear attention)
keep one latent row of 512 coordinates per token.  The text geometry is the published config
(benchmarks/microbench/glm53-flash-packed/model-config.json): `kv_lora_rank` 512 with no RoPE part
(`qk_rope_head_dim` 0, `mla_use_nope`), 64 heads of `qk_head_dim` 256, indexer top-k 2048.

* Native row: 512 raw E4M3 codes of the normalized latent (no scale), 512 bytes.
* Packed row, two planes: the 256 largest-|raw| coordinates' E4M3 codes in ascending coordinate order
  (256 bytes) and eight uint64 bitmap words (64 bytes); selection precedes the RMSNorm, which then runs
  over the kept coordinates (mean over all 512).

The arithmetic is the one of the V4 codec (`packmla.formats.codec`): the RMSNorm's sum of squares in
the store kernels' warp order, y = bf16((x r) w), codes = E4M3 round-to-nearest-even saturating at 448.
The reference does not state the bitmap's bit order; packmla uses LSB-first words (bit b of word w marks
coordinate 64 w + b), as for its V4 Packed rows.  K = V = the row; attention has no sink and no RoPE.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import codec

LATENT_DIM = 512
NATIVE_ROW_BYTES = 512
PACKED_KEEP = 256
BITMAP_WORDS = 8
PACKED_ROW_BYTES = PACKED_KEEP + 8 * BITMAP_WORDS  # 320
E4M3_MAX = 448.0


@dataclass(frozen=True)
class GLMGeometry:
    """The text geometry of GLM-5.3-Flash that the MLA KV and the decode kernel depend on."""

    num_layers: int = 45
    mla_layers: tuple = tuple(range(3, 45, 4))  # 3, 7, ..., 43: eleven DSA layers
    num_heads: int = 64
    kv_lora_rank: int = 512
    qk_head_dim: int = 256
    v_head_dim: int = 256
    index_topk: int = 2048
    index_head_dim: int = 128
    index_kpool: int = 4
    hidden_size: int = 4096

    @property
    def softmax_scale(self) -> float:
        return 1.0 / math.sqrt(self.qk_head_dim)


GLM53 = GLMGeometry()


def _e4m3(y: torch.Tensor) -> torch.Tensor:
    return y.to(torch.float32).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def native_encode(raw: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 latent rows [R, 512] (before the norm) -> Native rows uint8 [R, 512]."""
    return _e4m3(codec.rms_normalize(raw.to(torch.float32), weight, eps)).contiguous()


def packed_encode(raw: torch.Tensor, weight: torch.Tensor, eps: float,
                  mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 latent rows [R, 512] -> (values uint8 [R, 256], bitmap int64 [R, 8])."""
    raw = raw.to(torch.float32)
    if mask is None:
        mask = codec.topmag_mask(raw, PACKED_KEEP)
    if not bool((mask.sum(-1) == PACKED_KEEP).all()):
        raise ValueError(f"mask must keep exactly {PACKED_KEEP} coordinates per row")
    y = codec.rms_normalize(raw.masked_fill(~mask, 0.0), weight, eps)
    codes = _e4m3(y)
    return codes[mask].view(raw.shape[0], PACKED_KEEP).contiguous(), codec.bitmap_from_mask(mask)


def native_decode(rows: torch.Tensor) -> torch.Tensor:
    """Native rows [R, 512] -> fp32 [R, 512]."""
    return rows.contiguous().view(torch.float8_e4m3fn).to(torch.float32)


def native_from_packed(values: torch.Tensor, bitmap: torch.Tensor) -> torch.Tensor:
    """Adapter: Packed rows -> the Native rows holding the survivors (dropped coordinates code 0).  A row
    whose bitmap does not hold 256 bits (one never stored is all zero) maps its first set bits to its values
    in order; bits past the 256th read code 0."""
    mask = codec.mask_from_bitmap(bitmap)
    rank = mask.to(torch.int64).cumsum(-1) - 1
    kept = mask & (rank < PACKED_KEEP)
    gathered = values.to(torch.uint8).gather(1, rank.clamp(0, PACKED_KEEP - 1))
    return torch.where(kept, gathered, torch.zeros_like(gathered)).contiguous()


def packed_decode(values: torch.Tensor, bitmap: torch.Tensor) -> torch.Tensor:
    """Packed rows -> fp32 [R, 512] (dropped coordinates 0)."""
    return native_decode(native_from_packed(values, bitmap))


def sparse_decode_reference(q: torch.Tensor, kv_rows: list[torch.Tensor], scale: float):
    """fp32 reference: q [B, H, 512]; kv_rows[b] = [N_b, 512] decoded rows (K = V, no sink, no RoPE).
    Returns (out bf16 [B, H, 512], lse fp32 [B, H])."""
    from ..oracle.attention import attend

    H = q.shape[1]
    no_sink = torch.full((H,), float("-inf"))
    outs, lses = [], []
    for b in range(q.shape[0]):
        if kv_rows[b].shape[0] == 0:  # no rows and no sink: a zero output, LSE -inf (as the kernel)
            outs.append(torch.zeros(H, LATENT_DIM, dtype=torch.bfloat16))
            lses.append(torch.full((H,), float("-inf")))
            continue
        o, lse = attend(q[b].float(), kv_rows[b].float(), no_sink, scale)
        outs.append(o.to(torch.bfloat16))
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def bytes_per_token(fmt: str, geometry: GLMGeometry = GLM53, index_bytes: int = 132) -> int:
    """Per-token bytes of the MLA layers' KV (rows plus `index_bytes` of indexer key per layer: 128 FP8
    codes and an fp32 scale by default).  KDA state is per request and not counted."""
    row = {"native": NATIVE_ROW_BYTES, "direct": PACKED_ROW_BYTES}[fmt]
    return len(geometry.mla_layers) * (row + index_bytes)

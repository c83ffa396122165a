"""Dense projections with MXFP8 weights: y = x W^T.

Weights are stored as MXFP8: E4M3 codes [.., N, K] and one UE8M0 scale per 32 values along K (the rule of
`codec.ue8m0_exponent`, as for the MoE activations).  On CUDA `mx_linear` quantizes the activations per
token to MXFP8 and runs the block-scaled tcgen05 GEMM of csrc/dense_mx.cu (weights streamed as the
256-row operand; K splits for decode-sized token counts).  On CPU it computes the same arithmetic in fp32:
dequantized weights times MXFP8-rounded activations, rounded to BF16 - the oracle of the kernel.

Reference behaviour: the reference's dense layers are FP8 E4M3 weights with FP8 activations (SGLang's FP8
linear); MXFP8 is the Blackwell-native block-scaled form of that (power-of-two scales per 32 instead of fp32
scales per 128 x 128 block).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..formats import codec
from ._ext import error_word, ext

TILE_N = 256
GROUP_K = 128


@dataclass
class MxWeight:
    """MXFP8 weight of `batch` independent [N, K] matrices."""

    codes: torch.Tensor   # uint8 [batch, N, K] E4M3
    scales: torch.Tensor  # uint8 [batch, N, K / 32] UE8M0 (exponent + 127)
    sf_img: torch.Tensor  # uint8 [batch, N/256 tiles, K/128, 256, 4]: the kernel's per-tile, per-group blocks

    @property
    def batch(self) -> int:
        return self.codes.shape[0]

    @property
    def n(self) -> int:
        return self.codes.shape[1]

    @property
    def k(self) -> int:
        return self.codes.shape[2]

    def nbytes(self) -> int:
        return self.codes.numel() + self.scales.numel() + self.sf_img.numel()


def _arrange_scales(scales: torch.Tensor) -> torch.Tensor:
    """[batch, N, K/32] -> [batch, tiles, K/128, 256, 4] (rows past N padded with scale 2^0)."""
    b, n, kb = scales.shape
    tiles = -(-n // TILE_N)
    pad = torch.full((b, tiles * TILE_N, kb), 127, dtype=torch.uint8, device=scales.device)
    pad[:, :n] = scales
    return pad.view(b, tiles, TILE_N, kb // 4, 4).permute(0, 1, 3, 2, 4).contiguous()


def quantize_weight(w: torch.Tensor) -> MxWeight:
    """BF16/fp32 weight [N, K] or [batch, N, K] -> MXFP8 (per 32 along K, UE8M0 scale, E4M3 codes)."""
    if w.dim() == 2:
        w = w[None]
    b, n, k = w.shape
    if k % GROUP_K:
        raise ValueError(f"K = {k} must be a multiple of {GROUP_K}")
    codes = torch.empty(b, n, k, dtype=torch.uint8, device=w.device)
    scales = torch.empty(b, n, k // 32, dtype=torch.uint8, device=w.device)
    step = max(1, (1 << 26) // max(1, k))  # rows per chunk: bounded fp32 temporaries
    for bi in range(b):
        for r0 in range(0, n, step):
            blk = w[bi, r0:r0 + step].float().reshape(-1, k // 32, 32)
            e = codec.ue8m0_exponent(blk.abs().amax(-1))
            codes[bi, r0:r0 + step] = codec.e4m3_encode(blk * codec.exp2_int(-e)[..., None]).reshape(-1, k)
            scales[bi, r0:r0 + step] = (e + 127).to(torch.uint8)
    return MxWeight(codes, scales, _arrange_scales(scales))


def dequantize(w: MxWeight) -> torch.Tensor:
    """fp32 [batch, N, K] (exact: E4M3 x 2^e)."""
    b, n, k = w.codes.shape
    v = codec.e4m3_decode(w.codes).view(b, n, k // 32, 32)
    e = w.scales.to(torch.int32) - 127
    return (v * codec.exp2_int(e)[..., None]).view(b, n, k)


def mx_round(x: torch.Tensor) -> torch.Tensor:
    """MXFP8 round trip of x [..., K] in fp32: the activation quantization of the kernel."""
    shp = x.shape
    xb = x.float().reshape(*shp[:-1], shp[-1] // 32, 32)
    e = codec.ue8m0_exponent(xb.abs().amax(-1))
    q = codec.e4m3_decode(codec.e4m3_encode(xb * codec.exp2_int(-e)[..., None]))
    return (q * codec.exp2_int(e)[..., None]).reshape(shp)


def choose_splits(tokens: int, n: int, k: int, batch: int = 1, num_sms: int = 148) -> int:
    """K splits per 256-row tile: the count that minimizes the busiest CTA's work (units per CTA x (128-K
    groups per unit + 1 for a unit's pipeline fill and epilogue)), the smaller count on ties.  One split above 128 tokens, and when the tiles alone
    cover the SMs (the fp32 reductions of a split would cost more than the last wave's imbalance)."""
    tiles = batch * -(-n // TILE_N)
    if tokens > 128 or tiles >= num_sms:
        return 1
    groups = k // GROUP_K
    best, best_cost = 1, None
    for s in range(1, groups + 1):
        cost = math.ceil(tiles * s / num_sms) * (math.ceil(groups / s) + 1)
        if best_cost is None or cost < best_cost:
            best, best_cost = s, cost
    return best


A_IMG_MAX, A_SF_MAX = 65536, 16384  # the kernel's shared-memory activation image and its scale words


def fused_quant(tokens: int, k: int, splits: int) -> bool:
    """Whether the GEMM quantizes the activations itself (the rule of dense_mx_fused_quant)."""
    tp = (tokens + 7) // 8 * 8
    g_unit = -(-(k // GROUP_K) // splits)
    return tp <= 128 and tp * 128 * g_unit <= A_IMG_MAX and tp * 4 * g_unit <= A_SF_MAX


def call_needs(tokens: int, n: int, k: int, batch: int = 1, num_sms: int = 148,
               splits: int | None = None) -> tuple[int, int, int]:
    """(activation-image bytes, partial floats, tile counters) one `mx_linear` call needs."""
    s = splits or choose_splits(tokens, n, k, batch, num_sms)
    tp = (tokens + 7) // 8 * 8
    tiles = -(-n // TILE_N)
    a_bytes = 0 if fused_quant(tokens, k, s) else batch * (k // GROUP_K) * tp * 128
    if s > 1:
        return a_bytes, batch * s * tp * tiles * TILE_N, batch * tiles
    return a_bytes, 0, 0


class DenseWorkspace:
    """Activation images (prefill-sized calls), split-K partials and tile counters of `mx_linear` (stable
    pointers: safe to capture in CUDA graphs).  The counters are zero between calls (the kernel restores
    them).  `for_calls` sizes one workspace for a set of calls (tokens, N, K, batch) run one at a time."""

    def __init__(self, a_bytes: int, part_floats: int, counters: int, device, num_sms: int = 148):
        self.num_sms = num_sms
        self.a_img = torch.empty(max(16, a_bytes), dtype=torch.uint8, device=device)
        self.a_sf = torch.empty(max(4, a_bytes // 128), dtype=torch.int32, device=device)
        self.part = torch.empty(max(4, part_floats), dtype=torch.float32, device=device)
        self.counters = torch.zeros(max(1, counters), dtype=torch.int32, device=device)

    @classmethod
    def for_calls(cls, calls, device, num_sms: int = 148) -> "DenseWorkspace":
        need = [call_needs(t, n, k, b, num_sms) for t, n, k, b in calls]
        return cls(max(x[0] for x in need), max(x[1] for x in need), max(x[2] for x in need), device, num_sms)

    def holds(self, a_bytes: int, part_floats: int, counters: int) -> bool:
        return a_bytes <= self.a_img.numel() and part_floats <= self.part.numel() and counters <= self.counters.numel()

    def fits(self, tokens: int, k: int, n: int, batch: int, splits: int | None = None) -> bool:
        return self.holds(*call_needs(tokens, n, k, batch, self.num_sms, splits))


_WS: dict[int, DenseWorkspace] = {}
_NUM_SMS: dict[int, int] = {}


def _workspace(need: tuple[int, int, int], device) -> DenseWorkspace:
    """The per-device workspace of calls that bring none (grown when a call needs more; not for use
    inside CUDA-graph capture)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None or not ws.holds(*need):
        a, part, cnt = need
        if ws is not None:
            a, part, cnt = max(a, ws.a_img.numel()), max(part, ws.part.numel()), max(cnt, ws.counters.numel())
        ws = DenseWorkspace(a, part, cnt, device, _NUM_SMS.get(idx, 148))
        _WS[idx] = ws
    return ws


def mx_linear(x: torch.Tensor, w: MxWeight, out: torch.Tensor | None = None,
              workspace: DenseWorkspace | None = None, splits: int | None = None) -> torch.Tensor:
    """x [T, K] (w.batch == 1) or [batch, T, K] BF16 -> y [T, N] / [batch, T, N] BF16."""
    squeeze = x.dim() == 2
    x3 = x[None] if squeeze else x
    b, t, k = x3.shape
    if b != w.batch or k != w.k:
        raise ValueError(f"x {tuple(x.shape)} does not match weight [{w.batch}, {w.n}, {w.k}]")
    if not x3.is_cuda:
        y = (mx_round(x3) @ dequantize(w).transpose(1, 2)).to(torch.bfloat16)
        if out is not None:
            out.copy_(y[0] if squeeze else y)
            return out
        return y[0] if squeeze else y
    if x3.stride(2) != 1:
        x3 = x3.contiguous()
    dev = x3.device
    if out is None:
        y3 = torch.empty(b, t, w.n, dtype=torch.bfloat16, device=dev)
    else:
        y3 = out[None] if squeeze else out
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    s = splits or choose_splits(t, w.n, k, b, _NUM_SMS[idx])
    need = call_needs(t, w.n, k, b, _NUM_SMS[idx], s)
    if workspace is not None:
        if not workspace.holds(*need):
            raise ValueError(f"dense workspace too small for {b} x [{t}, {k}] x [{w.n}, {k}] at {s} splits")
        ws = workspace
    else:
        ws = _workspace(need, dev)
    ext().dense_mx(x3, w.codes, w.sf_img, y3, ws.a_img, ws.a_sf, ws.part, ws.counters, int(s), error_word(dev))
    return y3[0] if squeeze else y3

"""Sparse-attention indexer: FP8 index keys and per-query top-k C4 record selection.

score(b, r) = sum_h w[b, h] * relu(q[b, h] . k[r]) over records r < count[b]; the top-k records
(ties: lower record index first) are returned in ascending record order as physical slots and
RoPE rows (4 r), padded with slot -1.

Storage: keys[row] holds 128 E4M3 codes with its 16-byte units XOR-swizzled by (row % 8); scales[row]
= amax / 448.  Queries are quantized to E4M3 per head (amax / 448) inside the scorer, with the
per-head scale folded into w (relu is positively homogeneous).

CUDA: csrc/indexer.cu (tcgen05 kind::f8f6f4 logits + radix-select top-k).  CPU: the same
arithmetic in PyTorch (test oracle).
"""
from __future__ import annotations

import torch

from ..formats import abi
from ._ext import error_word, ext

E4M3_MAX = abi.E4M3_MAX


def _swizzle_units(rows: torch.Tensor) -> torch.Tensor:
    """Permutation of the 8 16-byte units of each row: stored unit u' holds logical unit u' ^ (row % 8)."""
    return torch.arange(8, device=rows.device)[None, :] ^ (rows[:, None] % 8)


def index_key_store(kraw: torch.Tensor, slots: torch.Tensor, keys: torch.Tensor, scales: torch.Tensor) -> None:
    if kraw.is_cuda:
        ext().index_key_store(kraw.float().contiguous(), slots.to(torch.int64).contiguous(), keys, scales,
                              error_word(kraw.device))
        return
    ok = slots >= 0
    if not bool(ok.any()):
        return
    k = kraw[ok].float()
    s = slots[ok].long()
    amax = k.abs().amax(-1, keepdim=True)
    sc = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    codes = (k * (1.0 / sc)).to(torch.float8_e4m3fn).view(torch.uint8).view(-1, 8, 16)
    perm = _swizzle_units(s)
    stored = torch.gather(codes, 1, perm[:, :, None].expand(-1, -1, 16))
    keys[s] = stored.reshape(-1, 128)
    scales[s] = sc[:, 0]


def read_keys(keys: torch.Tensor, scales: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """Dequantized fp32 keys [..., 128] of physical rows (any shape), undoing the unit swizzle."""
    flat = rows.reshape(-1).long()
    st = keys[flat].view(-1, 8, 16)
    logical = torch.gather(st, 1, _swizzle_units(flat)[:, :, None].expand(-1, -1, 16)).reshape(-1, 128)
    vals = logical.view(torch.float8_e4m3fn).float() * scales[flat][:, None]
    return vals.reshape(*rows.shape, 128)


def quantize_queries(q: torch.Tensor, w: torch.Tensor):
    """Per-head E4M3 queries (as fp32 values) and weights with the head scale folded in."""
    qf = q.float()
    amax = qf.abs().amax(-1, keepdim=True)
    qs = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q8 = (qf * (1.0 / qs)).to(torch.float8_e4m3fn).float()
    return q8, w.float() * qs[..., 0]


def index_select(q: torch.Tensor, w: torch.Tensor, keys: torch.Tensor, scales: torch.Tensor, phys: torch.Tensor,
                 count: torch.Tensor, R: int, topk: int):
    """q [B, H, 128] bf16, w [B, H] fp32, phys [B, >=R] int32, count [B] int64 -> (slots, pos) int32 [B, topk]."""
    B = q.shape[0]
    dev = q.device
    if q.is_cuda:
        scores = torch.empty(B, R, dtype=torch.float32, device=dev)
        slots = torch.empty(B, topk, dtype=torch.int32, device=dev)
        pos = torch.empty(B, topk, dtype=torch.int32, device=dev)
        ext().index_select(q.contiguous(), w.float().contiguous(), keys, scales, phys, count.to(torch.int64).contiguous(),
                           int(R), scores, slots, pos, error_word(dev))
        return slots, pos
    q8, w2 = quantize_queries(q, w)
    ph = phys[:, :R].long()
    k = read_keys(keys, scales, ph.clamp(min=0))  # [B, R, 128] (scale applied)
    s = torch.relu(torch.einsum("bhd,brd->bhr", q8, k))
    score = (s * w2[:, :, None]).sum(1)
    r = torch.arange(R, device=dev)
    visible = (r[None] < count[:, None]) & (ph >= 0)
    score = torch.where(visible, score, torch.full_like(score, float("-inf")))
    kk = min(topk, R)
    order = torch.sort(score, dim=1, descending=True, stable=True).indices[:, :kk]
    chosen = torch.sort(order, dim=1).values
    vals = score.gather(1, chosen)
    sl = torch.where(vals > float("-inf"), ph.gather(1, chosen), torch.full_like(chosen, -1))
    out_s = torch.full((B, topk), -1, dtype=torch.int32, device=dev)
    out_p = torch.zeros((B, topk), dtype=torch.int32, device=dev)
    out_s[:, :kk] = sl.int()
    out_p[:, :kk] = (chosen * abi.C4_RATIO).int()
    return out_s, out_p

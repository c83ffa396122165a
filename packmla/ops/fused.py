"""Fused element-wise / reduction ops of the decode step (csrc/fused_ops.cu); PyTorch on CPU."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..formats import abi
from ._ext import ext


def add_rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, d: torch.Tensor | None = None,
                dfp32: torch.Tensor | None = None, inplace: bool = False):
    """Returns (x_new, h): x_new = bf16(x + d + dfp32) (x itself if no addend), h = bf16(rmsnorm(x_new) * w)."""
    has_add = d is not None or dfp32 is not None
    if x.is_cuda and x.shape[1] % 2 == 0 and x.shape[1] <= 8192:
        h = torch.empty_like(x)
        x_out = (x if inplace else torch.empty_like(x)) if has_add else None
        ext().add_rmsnorm(x, d, dfp32, x_out, w, float(eps), h)
        return (x_out if has_add else x), h
    xf = x.float()
    if d is not None:
        xf = xf + d.float()
    if dfp32 is not None:
        xf = xf + dfp32.float()
    if has_add:
        xn = xf.to(torch.bfloat16)
        xf = xn.float()
    else:
        xn = x
    h = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w).to(torch.bfloat16)
    return xn, h


def rope_q(q: torch.Tensor, pos: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Rotate coords 448..511 of q [B, H, 512] bf16 by freqs[pos] (in place on CUDA)."""
    if q.is_cuda:
        ext().rope_q(q, pos.to(torch.int64).contiguous(), freqs)
        return q
    fr = freqs[pos.long()]
    c, s = fr[:, None, :, 0], fr[:, None, :, 1]
    tail = q[..., abi.NOPE_DIM:].float().unflatten(-1, (abi.ROPE_PAIRS, 2))
    re, im = tail[..., 0], tail[..., 1]
    rot = torch.stack((re * c - im * s, re * s + im * c), -1).flatten(-2)
    return torch.cat((q[..., :abi.NOPE_DIM], rot.to(torch.bfloat16)), -1)


def comp_pool(proj: torch.Tensor, off: int, D: int, ape: torch.Tensor, state: torch.Tensor, req: torch.Tensor,
              pos: torch.Tensor) -> torch.Tensor:
    """One token per row of online-softmax pooling; returns raw fp32 [B, D] (valid where the group completes)."""
    ratio = ape.shape[0]
    if proj.is_cuda:
        raw = torch.empty(proj.shape[0], D, dtype=torch.float32, device=proj.device)
        ext().comp_pool(proj, off, D, ape, state, req.to(torch.int64).contiguous(), pos.to(torch.int64).contiguous(), raw)
        return raw
    val = proj[:, off:off + D].float()
    slot = pos.long() % ratio
    gate = proj[:, off + D:off + 2 * D].float() + ape[slot]
    st = state[req.long()]
    m, l, acc = st[:, 0], st[:, 1], st[:, 2]
    mn = torch.maximum(m, gate)
    a = torch.exp(m - mn)
    e = torch.exp(gate - mn)
    l2 = l * a + e
    acc2 = acc * a + e * val
    raw = acc2 / l2
    done = (slot == ratio - 1)[:, None]
    state[req.long()] = torch.stack((torch.where(done, torch.full_like(mn, float("-inf")), mn),
                                     torch.where(done, torch.zeros_like(l2), l2),
                                     torch.where(done, torch.zeros_like(acc2), acc2)), 1)
    return raw


def route_topk(logits: torch.Tensor, bias: torch.Tensor | None, k: int, scaling: float):
    """Sigmoid scores of bf16 logits; top-k of score + bias (ties: lower expert); weights normalized over the k."""
    T, E = logits.shape
    if logits.is_cuda and E <= 512:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        ext().route_topk(logits, bias, k, float(scaling), ids, w)
        return ids, w
    scores = torch.sigmoid(logits.float())
    key = scores + (bias if bias is not None else 0.0)
    order = torch.sort(key, dim=-1, descending=True, stable=True).indices[:, :k]
    w = scores.gather(1, order)
    return order.int(), w / w.sum(-1, keepdim=True) * scaling


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    I = gu.shape[1] // 2
    if gu.is_cuda:
        out = torch.empty(gu.shape[0], I, dtype=torch.bfloat16, device=gu.device)
        ext().silu_mul(gu, out)
        return out
    return (F.silu(gu[:, :I].float()) * gu[:, I:].float()).to(torch.bfloat16)

"""fp32 CPU reference for compressed-sparse MLA attention (SWA + CSA + sink).

Semantics (training/losses.py:121-126, :203-213; training/tests/test_integration.py:1621-1633):

* one latent KV head of width 512 shared by all query heads; K and V are the same
  rotated latent row;
* per query: logits over [SWA rows ; selected CSA rows] scaled by `scale`, plus one
  per-head sink logit that behaves as an extra row whose value is zero;
* output tail (coordinates 448..511) inverse-rotated with the query position's
  frequency, then rounded to BF16.  LSE is the natural log of the softmax
  denominator including the sink.
"""

from __future__ import annotations

import math

import torch

from ..formats import abi, codec


def attend(q: torch.Tensor, kv: torch.Tensor, sink: torch.Tensor, scale: float):
    """q [H,512], kv [N,512], sink [H] -> (o [H,512] fp32 unrotated, lse [H])."""
    q = q.to(torch.float32)
    kv = kv.to(torch.float32)
    logits = torch.cat((q @ kv.T * scale, sink.to(torch.float32)[:, None]), -1)
    m = logits.amax(-1, keepdim=True)
    p = (logits - m).exp()
    denom = p.sum(-1, keepdim=True)
    o = (p[:, :-1] @ kv) / denom
    lse = (m + denom.log()).squeeze(-1)
    return o, lse


def sparse_mla_decode(
    q: torch.Tensor,
    kv_rows: list[torch.Tensor],
    sink: torch.Tensor,
    scale: float,
    q_freqs: torch.Tensor,
):
    """Batch of queries: q [B,H,512]; kv_rows[b] = [N_b, 512] decoded rows; q_freqs [B,32].

    Returns (out bf16 [B,H,512], lse fp32 [B,H]).
    """
    outs, lses = [], []
    for b in range(q.shape[0]):
        o, lse = attend(q[b], kv_rows[b], sink, scale)
        o = codec.rotate_tail(o.to(torch.bfloat16).to(torch.float32), q_freqs[b].expand(o.shape[0], -1), inverse=True)
        outs.append(o.to(torch.bfloat16))
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def default_scale(dim: int = abi.LATENT_DIM) -> float:
    return 1.0 / math.sqrt(dim)

"""Sparse MLA decode attention over Native SWA rows and Native/Packed C4 rows.

CUDA: tcgen05 kernel + split combine (csrc/attention_decode.cu).
CPU: fp32 oracle (packmla/oracle/attention.py) over rows decoded by the codec.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..formats import abi, codec
from ..oracle import attention as oracle
from ._ext import CLUSTER_SPLITS, decode_uses_partials, error_word, ext
from .kv import native_pool_read

NUM_SMS_B200 = 148
TILE_ROWS = 128
HEAD_GROUP = 64


@dataclass
class PackedPlanes:
    values: torch.Tensor  # uint8 [rows, 256]
    bitmap: torch.Tensor  # int64 [rows, 8]
    scales: torch.Tensor  # uint8 [rows, 8]


_MAX_CLUSTERS: dict[int, dict[int, int]] = {}


def max_active_clusters(device=None) -> dict[int, int]:
    """Co-resident decode clusters of 2, 4 and 8 CTAs on `device` (queried once per device)."""
    idx = torch.cuda.current_device() if device is None else torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    got = _MAX_CLUSTERS.get(idx)
    if got is None:
        with torch.cuda.device(idx):
            got = {s: int(ext().decode_max_active_clusters(s)) for s in CLUSTER_SPLITS}
        _MAX_CLUSTERS[idx] = got
    return got


def choose_tiling(batch: int, heads: int, max_rows: int, num_sms: int = NUM_SMS_B200,
                  max_clusters: dict[int, int] | None = None) -> tuple[int, int]:
    """(KV splits per (query, head group), KV rows per tile).

    One CTA per SM, one wave.  A split count of 2, 4 or 8 makes the splits of a (query, head group) one
    thread-block cluster that merges its partials on chip; the smallest such size that gives every split at
    most one 128-row tile is taken if its clusters are co-resident (`max_clusters`: size -> clusters), else
    the largest that is.  More than 8 tiles with room for more than 8 splits: one tile per split through
    the partial buffers and the combine kernel.  One split writes the output directly."""
    groups = (heads + HEAD_GROUP - 1) // HEAD_GROUP
    work = max(1, batch * groups)
    tiles = max(1, math.ceil(max_rows / TILE_ROWS))
    if tiles == 1:
        return 1, TILE_ROWS
    fit = num_sms // work
    mc = max_clusters or {s: num_sms // s for s in CLUSTER_SPLITS}
    sizes = [s for s in CLUSTER_SPLITS if s <= fit and work <= mc.get(s, 0)]
    if tiles > CLUSTER_SPLITS[-1] and fit > CLUSTER_SPLITS[-1]:
        return min(tiles, fit), TILE_ROWS
    if not sizes:
        return 1, TILE_ROWS
    for s in sizes:
        if s >= tiles:
            return s, TILE_ROWS
    return sizes[-1], TILE_ROWS


def check_cluster_fit(batch: int, heads: int, splits: int, device) -> None:
    """A split count of 2, 4 or 8 launches one thread-block cluster per (query, head group); every launch
    the kernel has been validated with keeps all of them co-resident, so a count whose clusters would not
    all fit at once is refused (`choose_tiling` never picks one)."""
    if splits in CLUSTER_SPLITS:
        work = batch * ((heads + HEAD_GROUP - 1) // HEAD_GROUP)
        fit = max_active_clusters(device).get(splits, 0)
        if work > fit:
            raise ValueError(f"{work} clusters of {splits} CTAs exceed the {fit} co-resident on this device")


def choose_splits(batch: int, heads: int, max_rows: int, num_sms: int = NUM_SMS_B200,
                  max_clusters: dict[int, int] | None = None) -> int:
    return choose_tiling(batch, heads, max_rows, num_sms, max_clusters)[0]


class DecodeWorkspace:
    """Split-KV partials with stable pointers (safe to capture in CUDA graphs); empty when the splits merge
    inside a cluster or there is one split."""

    def __init__(self, batch: int, heads: int, splits: int, device, tile_rows: int = TILE_ROWS):
        self.splits = splits
        self.tile_rows = tile_rows
        n = batch * splits * heads if decode_uses_partials(splits) else 0
        self.part_o = torch.empty(n * abi.LATENT_DIM, dtype=torch.float32, device=device)
        self.part_ml = torch.empty(n * 2, dtype=torch.float32, device=device)


def sparse_mla_decode(
    q: torch.Tensor,
    swa_pool: torch.Tensor,
    swa_slots: torch.Tensor,
    swa_len: torch.Tensor,
    csa_slots: torch.Tensor,
    csa_pos: torch.Tensor,
    csa_len: torch.Tensor,
    freqs: torch.Tensor,
    sink: torch.Tensor,
    scale: float,
    q_pos: torch.Tensor,
    csa_pool: torch.Tensor | None = None,
    csa_planes: PackedPlanes | None = None,
    num_splits: int | None = None,
    workspace: DecodeWorkspace | None = None,
    out: torch.Tensor | None = None,
    lse: torch.Tensor | None = None,
    prof: torch.Tensor | None = None,
    csa_fp4: str | None = None,
):
    """q [B,H,512] bf16 (tail rotated by the query position) -> (out bf16 [B,H,512], lse fp32 [B,H]).

    SWA rows: Native records at `swa_slots` [B, W] (first `swa_len[b]` used; -1 = masked).
    C4 rows: `csa_slots` [B, K] physical records, `csa_pos` [B, K] token positions (RoPE rows
    for Packed), first `csa_len[b]` used.  Exactly one of csa_pool (Native pages) /
    csa_planes (Packed) is given.  With `csa_fp4` ("native" or "direct") csa_pool holds FP4 pages of the V4.1
    cache (packmla.formats.fp4: Native 288 B or Packed 224 B records, RoPE applied at store, so `csa_pos` is
    not read).  `freqs` is float32 [P, 32, 2].  `prof` (optional int64 [64] on the
    device) receives global-timer stamps of the first CTA's pipeline steps, for latency analysis.
    """
    if (csa_pool is None) == (csa_planes is None):
        raise ValueError("give exactly one of csa_pool (native) or csa_planes (packed)")
    if csa_fp4 not in (None, "native", "direct") or (csa_fp4 and csa_pool is None):
        raise ValueError("csa_fp4 is 'native' or 'direct' and reads csa_pool")
    B, H, _ = q.shape
    if not q.is_cuda:
        return _decode_cpu(q, swa_pool, swa_slots, swa_len, csa_slots, csa_pos, csa_len, freqs, sink, scale, q_pos,
                           csa_pool, csa_planes, csa_fp4)
    if num_splits is None:
        if workspace is not None:
            num_splits = workspace.splits
        else:
            num_splits = choose_splits(B, H, swa_slots.shape[1] + csa_slots.shape[1],
                                       max_clusters=max_active_clusters(q.device))
    check_cluster_fit(B, H, num_splits, q.device)
    if workspace is None or workspace.splits != num_splits:
        workspace = DecodeWorkspace(B, H, num_splits, q.device)
    if out is None:
        out = torch.empty(B, H, abi.LATENT_DIM, dtype=torch.bfloat16, device=q.device)
    if lse is None:
        lse = torch.empty(B, H, dtype=torch.float32, device=q.device)
    packed = csa_planes is not None
    dev = q.device
    native_pool = csa_pool if not packed else torch.empty(0, dtype=torch.uint8, device=dev)
    values = csa_planes.values if packed else torch.empty(0, 256, dtype=torch.uint8, device=dev)
    bitmap = csa_planes.bitmap if packed else torch.empty(0, 8, dtype=torch.int64, device=dev)
    scales = csa_planes.scales if packed else torch.empty(0, 8, dtype=torch.uint8, device=dev)
    ext().sparse_mla_decode(
        q, swa_pool, swa_slots, swa_len, packed, native_pool, values, bitmap, scales,
        csa_slots, csa_pos, csa_len, freqs, sink, float(scale), q_pos, int(num_splits),
        workspace.part_o, workspace.part_ml, out, lse, error_word(dev), prof,
        {None: 0, "native": 1, "direct": 2}[csa_fp4],
    )
    return out, lse


def gather_rows_cpu(swa_pool, swa_slots_b, n_swa, csa_slots_b, csa_pos_b, n_csa, freqs, csa_pool, csa_planes,
                    csa_fp4=None):
    """Decoded fp32 rows [N, 512] of one query (masked -1 entries dropped)."""
    rows = []
    s = swa_slots_b[:n_swa].long()
    s = s[s >= 0]
    if s.numel():
        rows.append(codec.native_decode(native_pool_read(swa_pool, s).cpu()))
    c = csa_slots_b[:n_csa].long()
    p = csa_pos_b[:n_csa].long()
    valid = c >= 0
    c, p = c[valid], p[valid]
    if c.numel():
        if csa_fp4 is not None:
            from ..formats import fp4

            pages = csa_pool.cpu().view(-1, fp4.page_bytes(csa_fp4))
            rows.append(fp4.gather_rows(pages, csa_fp4, c))
        elif csa_planes is None:
            rows.append(codec.native_decode(native_pool_read(csa_pool, c).cpu()))
        else:
            fr = torch.view_as_complex(freqs[p].float().contiguous()).cpu()
            rows.append(codec.packed_read(csa_planes.values[c].cpu(), csa_planes.bitmap[c].cpu(),
                                          csa_planes.scales[c].cpu(), fr))
    if not rows:
        return torch.zeros(0, abi.LATENT_DIM)
    return torch.cat(rows)


def _decode_cpu(q, swa_pool, swa_slots, swa_len, csa_slots, csa_pos, csa_len, freqs, sink, scale, q_pos, csa_pool,
                csa_planes, csa_fp4=None):
    B = q.shape[0]
    kv = []
    for b in range(B):
        kv.append(gather_rows_cpu(swa_pool, swa_slots[b], int(swa_len[b]), csa_slots[b], csa_pos[b], int(csa_len[b]),
                                  freqs, csa_pool, csa_planes, csa_fp4))
    qf = torch.view_as_complex(freqs[q_pos.long()].float().contiguous())
    return oracle.sparse_mla_decode(q.float(), kv, sink.float(), scale, qf)

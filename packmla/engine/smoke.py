"""Tiny end-to-end check on one GPU (used by the driver's smoke step)."""
from __future__ import annotations

import torch


def run_smoke(device: torch.device) -> None:
    from ..formats import abi, codec
    from ..ops import attention as attn_ops
    from ..ops import check_errors
    from ..ops import kv as kv_ops

    torch.manual_seed(0)
    freqs = kv_ops.freq_table_f32(codec.rope_table(4096)).to(device)
    w = torch.ones(512, device=device)
    rows = 256
    raw = torch.randn(rows, 512, device=device)
    pool = torch.zeros(4 * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=device)
    kv_ops.native_store(raw, w, 1e-6, torch.arange(rows, device=device), torch.arange(rows, device=device), freqs, pool)
    planes = attn_ops.PackedPlanes(torch.zeros(rows, 256, dtype=torch.uint8, device=device),
                                   torch.zeros(rows, 8, dtype=torch.int64, device=device),
                                   torch.zeros(rows, 8, dtype=torch.uint8, device=device))
    kv_ops.packed_store(raw, w, 1e-6, torch.arange(rows, device=device), planes.values, planes.bitmap, planes.scales)
    B, H = 2, 64
    q = torch.randn(B, H, 512, device=device).bfloat16()
    swa = torch.arange(128, device=device, dtype=torch.int32).repeat(B, 1)
    csa = torch.arange(128, 256, device=device, dtype=torch.int32).repeat(B, 1)
    out, lse = attn_ops.sparse_mla_decode(
        q, pool, swa, torch.full((B,), 128, dtype=torch.int32, device=device), csa, csa * 4,
        torch.full((B,), 128, dtype=torch.int32, device=device), freqs, torch.zeros(H, device=device),
        512 ** -0.5, torch.zeros(B, dtype=torch.int32, device=device), csa_planes=planes)
    torch.cuda.synchronize(device)
    check_errors(device)
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()

"""GLM-5.3 MLA ops: row store (Native 512 B / Packed 320 B), Adapter, and sparse decode.

CUDA tensors run the sm_100a kernels: `glm_store` / `glm_packed_to_native` (csrc/kv_store.cu) and the
tcgen05 sparse MLA decode kernel with its GLM row kinds (csrc/attention_decode.cu: Native rows expand as
raw E4M3 into the FP16 K tile, Packed rows through the bitmap prefix-count expansion of the V4 Packed
rows, without scales or RoPE).  CPU tensors run the oracle (`packmla.formats.glm`); both produce the same
row bytes.

Reference behaviour: the GLM-5.3-Flash candidate's producer (writes the row once, selection before the
RMSNorm), Adapter (Packed -> Native workspace) and TileLang Direct decode expanding 320 B rows in the
KV tile (third_party/README.md:444-465).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..formats import glm
from ._ext import error_word, ext


# Batches above this stay off the device: the GLM decode suite's first batch-32 case raised an illegal address
# on its first CUDA-graph replay (the same graph's eager launches had passed).  That launch used 32 clusters
# of 4 CTAs chosen without the device's co-resident cluster count (which `check_cluster_fit` now enforces);
# reading the code has not yet shown the mechanism.
MAX_DEVICE_BATCH = 24


@dataclass
class GLMPlanes:
    values: torch.Tensor  # uint8 [rows, 256]
    bitmap: torch.Tensor  # int64 [rows, 8]


def glm_store(raw: torch.Tensor, weight: torch.Tensor, eps: float, slots: torch.Tensor,
              pool: torch.Tensor | None = None, planes: GLMPlanes | None = None) -> None:
    """Write rows `raw` fp32 [R, 512] (the latent before the norm) at `slots` (-1 = skip) of a Native pool
    uint8 [rows, 512] or of Packed planes."""
    if (pool is None) == (planes is None):
        raise ValueError("give exactly one of pool (native) or planes (packed)")
    if raw.is_cuda:
        e = torch.empty(0, dtype=torch.uint8, device=raw.device)
        ext().glm_store(raw, weight, float(eps), slots.to(torch.int64), planes is not None,
                        pool if pool is not None else e.view(0, 512),
                        planes.values if planes is not None else e.view(0, 256),
                        planes.bitmap if planes is not None else torch.empty(0, 8, dtype=torch.int64, device=raw.device),
                        error_word(raw.device))
        return
    keep = slots >= 0
    if not bool(keep.any()):
        return
    idx = slots[keep].long()
    if planes is None:
        pool[idx] = glm.native_encode(raw[keep], weight, eps)
    else:
        v, b = glm.packed_encode(raw[keep], weight, eps)
        planes.values[idx] = v
        planes.bitmap[idx] = b


def glm_packed_to_native(planes: GLMPlanes, rows: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Adapter: Native rows uint8 [R, 512] of the Packed rows `rows` (-1: a zero row)."""
    dev = planes.values.device
    if out is None:
        out = torch.empty(rows.numel(), glm.NATIVE_ROW_BYTES, dtype=torch.uint8, device=dev)
    if planes.values.is_cuda:
        ext().glm_packed_to_native(planes.values, planes.bitmap, rows.to(torch.int64), out, error_word(dev))
        return out
    r = rows.long()
    valid = r >= 0
    out.zero_()
    if bool(valid.any()):
        out[valid] = glm.native_from_packed(planes.values[r[valid]], planes.bitmap[r[valid]])
    return out


def glm_sparse_decode(q: torch.Tensor, slots: torch.Tensor, lens: torch.Tensor, scale: float | None = None,
                      pool: torch.Tensor | None = None, planes: GLMPlanes | None = None,
                      num_splits: int | None = None, workspace=None, out: torch.Tensor | None = None,
                      lse: torch.Tensor | None = None):
    """q bf16 [B, H, 512] (absorbed queries) over the rows `slots` int32 [B, K] (first `lens[b]` used,
    -1 masked) of a Native pool or Packed planes -> (out bf16 [B, H, 512], lse fp32 [B, H])."""
    from .attention import DecodeWorkspace, check_cluster_fit, choose_splits, max_active_clusters

    if (pool is None) == (planes is None):
        raise ValueError("give exactly one of pool (native) or planes (packed)")
    scale = glm.GLM53.softmax_scale if scale is None else scale
    B, H, _ = q.shape
    if q.is_cuda and B > MAX_DEVICE_BATCH:
        raise ValueError(f"GLM decode on the device is limited to batch {MAX_DEVICE_BATCH}: a batch-32 case raised "
                         "an illegal address under CUDA-graph replay and stays off the GPU until its cause is found")
    if not q.is_cuda:
        rows = []
        for b in range(B):
            s = slots[b, :int(lens[b])].long()
            s = s[s >= 0]
            rows.append(glm.native_decode(pool[s]) if planes is None
                        else glm.packed_decode(planes.values[s], planes.bitmap[s]))
        return glm.sparse_decode_reference(q, rows, scale)
    if num_splits is None:
        num_splits = workspace.splits if workspace is not None else choose_splits(
            B, H, slots.shape[1], max_clusters=max_active_clusters(q.device))
    check_cluster_fit(B, H, num_splits, q.device)
    if workspace is None or workspace.splits != num_splits:
        workspace = DecodeWorkspace(B, H, num_splits, q.device)
    if out is None:
        out = torch.empty(B, H, glm.LATENT_DIM, dtype=torch.bfloat16, device=q.device)
    if lse is None:
        lse = torch.empty(B, H, dtype=torch.float32, device=q.device)
    dev = q.device
    e8 = torch.empty(0, dtype=torch.uint8, device=dev)
    ext().glm_sparse_decode(
        q, 1 if planes is None else 2, pool if pool is not None else e8.view(0, 512),
        planes.values if planes is not None else e8.view(0, 256),
        planes.bitmap if planes is not None else torch.empty(0, 8, dtype=torch.int64, device=dev),
        slots, lens, float(scale), int(num_splits), workspace.part_o, workspace.part_ml, out, lse, error_word(dev))
    return out, lse

"""Reference math for training and evaluation, built on packmla's fp32 oracle.

The reference loads these functions from its SGLang fork's calibration runner (`calibrate.py`:
normalize / attention / rotate / decode_native / atomic_json / reference()) and its
reference codec (`srt/remnant/reference.py`: pack_rows_ref / unpack_rows_ref / topmag_keep_mask /
_ue8m0_quantize).  packmla's codec (packmla.formats.codec) is the byte-exact oracle of its own
store kernels, so training, evaluation and serving share one codec.
"""
from __future__ import annotations

import hashlib
import json
import os
import tempfile
from pathlib import Path

import torch

from ..formats import abi, codec
from ..oracle import attention as oracle


class Math:
    """Attention math of a captured decode query."""

    @staticmethod
    def rotate(x: torch.Tensor, freqs: torch.Tensor, inverse: bool = False) -> torch.Tensor:
        """Rotate the 64-wide tail of [..., 512] rows by complex64 freqs [..., 32] (broadcast)."""
        fr = freqs.to(torch.complex64)
        if fr.dim() < x.dim():
            fr = fr.expand(*x.shape[:-1], abi.ROPE_PAIRS)
        return codec.rotate_tail(x, fr, inverse)

    @staticmethod
    def attention(q: torch.Tensor, kv: torch.Tensor, sink: torch.Tensor, scale: float):
        """q [H,512], kv [N,512] (K = V = rotated latent rows), per-head sink -> (o [H,512], lse [H])."""
        return oracle.attend(q, kv, sink, scale)

    @staticmethod
    def normalize(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
        return codec.rms_normalize(x, weight, eps)

    @staticmethod
    def decode_native(records: torch.Tensor) -> torch.Tensor:
        return codec.native_decode(records)

    @staticmethod
    def atomic_json(path: Path, obj) -> None:
        """Write JSON to a temporary file beside `path`, fsync, then rename over it."""
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", dir=path.parent)
        try:
            with os.fdopen(fd, "w") as f:
                json.dump(obj, f, indent=2, sort_keys=True)
                f.flush()
                os.fsync(f.fileno())
            os.replace(tmp, path)
        except BaseException:
            if os.path.exists(tmp):
                os.unlink(tmp)
            raise


class Reference:
    """The Packed codec as the training code sees it (rows in, planes / dense rows out)."""

    @staticmethod
    def pack_rows_ref(raw, mask, weight, eps):
        return codec.packed_encode(raw, weight, eps, mask=mask)

    @staticmethod
    def unpack_rows_ref(values, bitmap, scales):
        return codec.packed_decode(values, bitmap, scales)

    @staticmethod
    def topmag_keep_mask(scores: torch.Tensor, fraction: float) -> torch.Tensor:
        return codec.topmag_mask(scores, int(round(fraction * abi.LATENT_DIM)))

    @staticmethod
    def _ue8m0_quantize(y: torch.Tensor):
        """bf16-valued [R,512] -> (E4M3 values as fp32 codes' values, UE8M0 codes [R,8])."""
        codes, scales = codec.quantize_tiles(y.float(), abi.NUM_TILES)
        return codec.e4m3_decode(codes).reshape(y.shape), scales


def reference() -> Reference:
    return Reference()


def file_sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(8 << 20), b""):
            h.update(block)
    return h.hexdigest()

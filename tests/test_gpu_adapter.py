"""Adapter kernel (csrc/adapter.cu): Packed planes -> Native records, byte-exact against the CPU oracle."""
import pytest
import torch

from packmla.formats import abi, codec
from packmla.ops import kv as kv_ops
from packmla.ops._ext import check_errors

pytestmark = pytest.mark.gpu


def _planes(n, seed):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(n, 512, generator=g) * torch.linspace(0.01, 40, 512)
    w = torch.rand(512, generator=g) + 0.5
    masks = [codec.topmag_mask(raw)]
    # extreme bitmaps: first half, second half, alternating coordinates
    m = torch.zeros(3, 512, dtype=torch.bool)
    m[0, :256] = True
    m[1, 256:] = True
    m[2, ::2] = True
    vals, bits, sc = codec.packed_encode(raw, w, 1e-6)
    v2, b2, s2 = codec.packed_encode(raw[:3], w, 1e-6, mask=m)
    return torch.cat((vals, v2)), torch.cat((bits, b2)), torch.cat((sc, s2))


def test_packed_to_native_matches_oracle(cuda):
    n = 200
    vals, bits, sc = _planes(n, 1)
    rows = vals.shape[0]
    table = codec.rope_table(4096)
    freqs = torch.stack((table.real, table.imag), -1).float().contiguous()
    g = torch.Generator().manual_seed(2)
    src = torch.randint(0, rows, (300,), generator=g, dtype=torch.int32)
    pos = torch.randint(0, 4096, (300,), generator=g, dtype=torch.int32)
    dst = torch.randperm(320, generator=g)[:300].long()
    dst[5] = -1  # skipped destination
    pages = 320 // abi.RECORDS_PER_PAGE
    out_cpu = torch.zeros(pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8)
    kv_ops.packed_to_native(vals, bits, sc, src, pos, freqs, out_cpu, dst)
    out_gpu = torch.zeros_like(out_cpu, device=cuda)
    kv_ops.packed_to_native(vals.to(cuda), bits.to(cuda), sc.to(cuda), src.to(cuda), pos.to(cuda), freqs.to(cuda),
                            out_gpu, dst.to(cuda))
    check_errors(cuda)
    assert torch.equal(out_gpu.cpu(), out_cpu)

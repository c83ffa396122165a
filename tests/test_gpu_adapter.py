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


@pytest.mark.parametrize("keep", [64, 192, 320, 448])
def test_packed_layouts_of_other_survivor_counts(cuda, keep):
    """Per-layer Packed layouts (K survivors, values planes of K bytes): the device store writes the CPU
    codec's planes byte for byte, ties included, and the reconstruction reads them back into the CPU
    oracle's Native records."""
    g = torch.Generator().manual_seed(keep)
    n = 150
    raw = torch.randn(n, 512, generator=g) * 2
    raw[0] = torch.round(raw[0] * 2) / 2  # magnitude ties at the selection boundary
    raw[1] = 1.0
    w = torch.rand(512, generator=g) + 0.25
    slots = torch.randperm(n + 7, generator=g)[:n]
    planes = [torch.full((n + 7, keep), 3, dtype=torch.uint8), torch.zeros(n + 7, 8, dtype=torch.int64),
              torch.zeros(n + 7, 8, dtype=torch.uint8)]
    gplanes = [t.to(cuda) for t in planes]
    kv_ops.packed_store(raw.to(cuda), w.to(cuda), 1e-6, slots.to(cuda), *gplanes)
    check_errors(cuda)
    kv_ops.packed_store(raw, w, 1e-6, slots, *planes)
    for a, b in zip(gplanes, planes):
        assert torch.equal(a.cpu(), b)
    table = codec.rope_table(4096)
    freqs = torch.stack((table.real, table.imag), -1).float().contiguous()
    src = slots[:100].int()
    pos = torch.randint(0, 4096, (100,), generator=g, dtype=torch.int32)
    dst = torch.arange(100, dtype=torch.int64)
    out_cpu = torch.zeros(2 * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8)
    kv_ops.packed_to_native(*planes, src, pos, freqs, out_cpu, dst)
    out_gpu = torch.zeros_like(out_cpu, device=cuda)
    kv_ops.packed_to_native(*gplanes, src.to(cuda), pos.to(cuda), freqs.to(cuda), out_gpu, dst.to(cuda))
    check_errors(cuda)
    assert torch.equal(out_gpu.cpu(), out_cpu)

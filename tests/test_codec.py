"""CPU tests of the record codec (the byte contract of every store/read kernel)."""
import math

import torch

from packmla.formats import abi, codec


def test_record_sizes():
    assert abi.NATIVE_RECORD_BYTES == 584 and abi.PACKED_RECORD_BYTES == 328
    assert abi.NATIVE_PAGE_BYTES % 16 == 0 and abi.NATIVE_DATA_BYTES % 16 == 0
    assert abi.packed_record_bytes(192) == 264


def test_ue8m0_rule_matches_log2_definition():
    vals = [0.0, 1e-6, 1e-4, 0.03125, 1.0, 447.0, 448.0, 448.5, 896.0, 896.01, 1e6]
    for v in vals:
        e = int(codec.ue8m0_exponent(torch.tensor([v], dtype=torch.float32)))
        assert e == math.ceil(math.log2(max(float(torch.tensor(v, dtype=torch.float32)), 1e-4) / 448)), v


def test_topmag_ties_keep_lower_coordinate():
    raw = torch.ones(1, 512)
    raw[0, 500] = 2.0
    m = codec.topmag_mask(raw, 256)
    assert m.sum() == 256 and m[0, 500] and m[0, :255].all() and not m[0, 255:500].any()


def test_bitmap_roundtrip_lsb_first():
    mask = torch.zeros(2, 512, dtype=torch.bool)
    mask[0, 0] = True
    mask[0, 63] = True
    mask[1, 64 * 7 + 5] = True
    words = codec.bitmap_from_mask(mask)
    assert words[0, 0].item() == (1 | -(1 << 63))
    assert words[1, 7].item() == 1 << 5
    assert torch.equal(codec.mask_from_bitmap(words), mask)


def test_packed_roundtrip_and_ascending_values():
    g = torch.Generator().manual_seed(0)
    raw = torch.randn(16, 512, generator=g)
    w = torch.rand(512, generator=g) + 0.5
    v, b, s = codec.packed_encode(raw, w, 1e-6)
    assert v.shape == (16, 256) and b.shape == (16, 8) and s.shape == (16, 8)
    mask = codec.mask_from_bitmap(b)
    assert torch.equal(mask, codec.topmag_mask(raw))
    dense = codec.packed_decode(v, b, s)
    sim = codec.simulated_packed_rows(raw, mask, w, 1e-6, codec.rope_table(1)[[0] * 16])
    fr = codec.rope_table(1)[[0] * 16]
    assert torch.equal(codec.packed_read(v, b, s, fr), sim)
    assert (dense[~mask] == 0).all()


def test_independent_192_survivor_derivation():
    """Constant rows, per-tile weights 2^t: derive BF16 values/scales from Python scalars."""
    eps = 1e-6
    raw = torch.ones(4, 512)
    weight = torch.tensor([2.0 ** t for t in range(8)]).repeat_interleave(64)
    mask = (torch.arange(512) % 8 >= 5).expand(4, -1)
    freqs = codec.rope_table(64)[torch.arange(4) * 4]
    expected = torch.zeros(4, 512)
    for t in range(8):
        normalized = float(torch.tensor((2.0 ** t) / math.sqrt(192 / 512 + eps)).bfloat16())
        scale = 2.0 ** math.ceil(math.log2(max(abs(normalized), 1e-4) / 448))
        code = torch.tensor(normalized / scale).to(torch.float8_e4m3fn).float()
        expected[:, t * 64:(t + 1) * 64] = (code * scale).bfloat16().float()
    expected.masked_fill_(~mask, 0)
    expected = codec.rotate_tail(expected, freqs).bfloat16().float()
    got = codec.simulated_packed_rows(raw, mask, weight, eps, freqs)
    assert torch.equal(got, expected)


def test_native_encode_layout():
    g = torch.Generator().manual_seed(1)
    raw = torch.randn(3, 512, generator=g)
    w = torch.ones(512)
    fr = codec.rope_table(16)[[0, 4, 8]]
    rec = codec.native_encode(raw, w, 1e-6, fr)
    assert rec.shape == (3, 584)
    assert (rec[:, 583] == 0).all()  # pad byte
    dec = codec.native_decode(rec)
    y = codec.rms_normalize(raw, w, 1e-6)
    assert torch.equal(dec[:, 448:], codec.rotate_tail(y, fr)[:, 448:].bfloat16().float())
    rel = (dec[:, :448] - y[:, :448]).norm() / y[:, :448].norm()
    assert rel < 0.05


def test_adapter_native_view_decodes_to_the_packed_read():
    """Re-quantizing exactly decoded Packed values is lossless: the Adapter's Native record decodes to
    the same rows a Direct reader sees."""
    g = torch.Generator().manual_seed(11)
    raw = torch.randn(40, 512, generator=g) * torch.linspace(0.01, 30, 512)
    raw[3] = 0  # all-zero row: every tile at the amax floor
    w = torch.rand(512, generator=g) + 0.5
    vals, bits, sc = codec.packed_encode(raw, w, 1e-6)
    ang = torch.rand(40, 32, generator=g) * 6.28
    fr = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    native = codec.native_from_packed(vals, bits, sc, fr)
    assert torch.equal(codec.native_decode(native), codec.packed_read(vals, bits, sc, fr))


def test_oracle_experiment_config():
    """CPU oracle experiment: byte accounting, mask geometry, Native close to unquantized rows, and the
    capacity ratio of Direct over Native."""
    from packmla.bench.oracle_experiment import run

    out = run(batch=2, heads=8, context=2048, topk=128)
    assert out["records"] == 512 and out["mask"] == {"rope_kept": 64, "nope_kept": 192}
    assert out["bytes"]["packed_layer"] == 512 * 328 and out["bytes"]["native_layer"] == 512 * 584
    assert out["relative_output_error"]["native_vs_exact"]["max"] < 0.05
    assert out["relative_output_error"]["topmag_vs_native"]["mean"] < out["relative_output_error"]["packed_vs_native"]["mean"]
    assert out["capacity_tokens_30GiB"]["ratio"] >= 1.21

"""CPU: property tests of the record codecs over generated rows (hypothesis).

Invariants: bitmaps round-trip any mask in both bit orders; Packed values are the Native-tile codes
of the kept coordinates in ascending order and decode to zero elsewhere; a decoded Packed row
quantizes each 64-wide tile within one E4M3 step of its RMS-normalised input; FP4 survivors are
exactly the top dequantized magnitudes and Packed FP4 equals the masked Native FP4 row.
"""
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from packmla.formats import abi, codec, fp4

SETTINGS = settings(max_examples=25, deadline=None, derandomize=True, database=None,
                    suppress_health_check=[HealthCheck.too_slow])


@st.composite
def rows(draw, n_max=4):
    n = draw(st.integers(1, n_max))
    seed = draw(st.integers(0, 2 ** 31 - 1))
    scale = draw(st.sampled_from([1e-3, 0.1, 1.0, 30.0]))
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, abi.LATENT_DIM, generator=g) * scale
    if draw(st.booleans()):  # heavy ties: quantize magnitudes to a few levels
        x = torch.round(x / scale * 2) * scale / 2
    if draw(st.booleans()):  # a zero tile
        t = draw(st.integers(0, abi.NUM_TILES - 1))
        x[:, t * 64:(t + 1) * 64] = 0
    return x


@st.composite
def masks(draw):
    n = draw(st.integers(1, 4))
    seed = draw(st.integers(0, 2 ** 31 - 1))
    g = torch.Generator().manual_seed(seed)
    return torch.rand(n, abi.LATENT_DIM, generator=g) < draw(st.floats(0.0, 1.0))


@SETTINGS
@given(masks())
def test_bitmaps_roundtrip_any_mask(mask):
    assert torch.equal(codec.mask_from_bitmap(codec.bitmap_from_mask(mask)), mask)
    assert torch.equal(fp4.mask_from_msb_bitmap(fp4.bitmap_msb_first(mask)), mask)
    # the two orders are bit reversals of each other within every word
    lsb = codec.bitmap_from_mask(mask)
    rev = codec.bitmap_from_mask(mask.view(-1, 8, 64).flip(-1).reshape(mask.shape))
    assert torch.equal(fp4.bitmap_msb_first(mask), rev) and lsb.shape == rev.shape


@SETTINGS
@given(rows())
def test_packed_values_are_ascending_kept_codes(x):
    w = torch.ones(abi.LATENT_DIM)
    values, bitmap, scales = codec.packed_encode(x, w, 1e-6)
    mask = codec.mask_from_bitmap(bitmap)
    assert bool((mask.sum(-1) == abi.PACKED_KEEP).all())
    y = codec.rms_normalize(x.masked_fill(~mask, 0.0), w, 1e-6)
    codes, sc = codec.quantize_tiles(y, abi.NUM_TILES)
    assert torch.equal(sc, scales)
    assert torch.equal(values, codes[mask].view(x.shape[0], abi.PACKED_KEEP))
    dec = codec.packed_decode(values, bitmap, scales)
    assert bool((dec[~mask] == 0).all())
    # within one E4M3 step (relative 2^-3 of the tile scale's binade) of the normalised input
    s = codec.exp2_int(scales.to(torch.int32) - abi.UE8M0_BIAS).repeat_interleave(64, -1)
    err = (dec - y.to(torch.bfloat16).float()).abs()[mask]
    assert bool((err <= (s * 32)[mask] + 1e-6).all())


@SETTINGS
@given(rows())
def test_topmag_keeps_the_largest(x):
    mask = codec.topmag_mask(x)
    a = x.abs()
    for r in range(x.shape[0]):
        kept, dropped = a[r][mask[r]], a[r][~mask[r]]
        assert float(kept.min()) >= float(dropped.max())


@SETTINGS
@given(rows())
def test_fp4_packed_is_masked_native(x):
    x = x.to(torch.bfloat16).float()
    codes, scales = fp4.native_encode(x)
    native = fp4.native_decode(codes, scales)
    pc, words, ps = fp4.packed_encode(x)
    mask = fp4.mask_from_msb_bitmap(words)
    assert bool((mask.sum(-1) == fp4.KEEP).all())
    assert torch.equal(fp4.packed_decode(pc, words, ps), native * mask)
    mag = native.abs()
    for r in range(x.shape[0]):
        assert float(mag[r][mask[r]].min()) >= float(mag[r][~mask[r]].max())
    # decoding is idempotent for groups whose scale is zero or a normal E4M3 value (>= 2^-6): the group
    # maximum then always encodes as 6, so the re-derived scale is the same.  Subnormal scales round
    # coarsely and may change.
    c2, s2 = fp4.native_encode(native)
    sv = scales.view(torch.float8_e4m3fn).float()
    normal = ((sv == 0) | (sv >= 2.0 ** -6)).repeat_interleave(16, -1)
    assert torch.equal(fp4.native_decode(c2, s2)[normal], native[normal])

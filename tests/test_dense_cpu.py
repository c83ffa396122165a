"""MXFP8 dense weight format and split choice (CPU)."""
import torch

from packmla.ops import dense as dense_ops


def test_scale_image_layout_matches_row_scales():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(2, 300, 512, generator=g)
    q = dense_ops.quantize_weight(w)
    assert q.codes.shape == (2, 300, 512) and q.scales.shape == (2, 300, 16)
    assert q.sf_img.shape == (2, 2, 4, 256, 4)
    # tile 1, group 3, row 10, block 2 <-> weight row 256 + 10, scale block 4 * 3 + 2
    assert int(q.sf_img[1, 1, 3, 10, 2]) == int(q.scales[1, 266, 14])
    assert int(q.sf_img[0, 1, 0, 200, 0]) == 127  # rows past N: scale 2^0


def test_cpu_linear_is_mxfp8_arithmetic():
    g = torch.Generator().manual_seed(2)
    w = torch.randn(64, 256, generator=g)
    x = torch.randn(5, 256, generator=g).bfloat16()
    q = dense_ops.quantize_weight(w)
    y = dense_ops.mx_linear(x, q)
    ref = (dense_ops.mx_round(x.float()) @ dense_ops.dequantize(q)[0].T).bfloat16()
    assert y.shape == (5, 64) and torch.equal(y, ref)


def test_choose_splits_covers_the_sms():
    assert dense_ops.choose_splits(8, 4096, 4096) > 1  # 16 tiles: split K
    assert dense_ops.choose_splits(8, 129280, 4096) == 1  # 505 tiles already cover the SMs
    assert dense_ops.choose_splits(300, 4096, 4096) == 1  # more than one token tile: no split
    s = dense_ops.choose_splits(8, 4352, 4096)
    assert 1 < s <= 32

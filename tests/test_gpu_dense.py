"""MXFP8 dense projections (csrc/dense_mx.cu) against the fp32 oracle of the same arithmetic."""
import pytest
import torch

from packmla.ops import check_errors
from packmla.ops import dense as dense_ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,T,K,N,splits", [
    (1, 8, 4096, 4352, None),    # decode FFN input projection: K splits
    (1, 40, 1024, 8192, None),   # q-LoRA up-projection width
    (1, 3, 8192, 4096, None),    # output projection (K = 8192)
    (8, 8, 4096, 1024, None),    # grouped projection (8 independent weights)
    (1, 300, 1024, 1000, None),  # prefill-sized: three token tiles, ragged last weight tile
    (1, 16, 2048, 4096, 1),      # forced single split
])
def test_mx_linear_matches_oracle(cuda, batch, T, K, N, splits):
    g = torch.Generator().manual_seed(T * 7 + K + N)
    w = torch.randn(batch, N, K, generator=g) * K ** -0.5
    x = torch.randn(batch, T, K, generator=g).bfloat16()
    wq = dense_ops.quantize_weight(w)
    ref = dense_ops.mx_linear(x, wq).float()  # CPU: fp32 arithmetic of the kernel, BF16 output
    wg = dense_ops.MxWeight(wq.codes.cuda(), wq.scales.cuda(), wq.sf_img.cuda())
    for _ in range(2):  # the split-K accumulator must be back to zero for the second call
        y = dense_ops.mx_linear(x.cuda(), wg, splits=splits)
        check_errors(cuda)
        torch.testing.assert_close(y.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_mx_weight_round_trip_is_close():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 256, generator=g)
    d = dense_ops.dequantize(dense_ops.quantize_weight(w))[0]
    rel = ((d - w).norm() / w.norm()).item()
    assert rel < 0.05  # E4M3: 3 mantissa bits

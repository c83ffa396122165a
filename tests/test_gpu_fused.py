"""Fused decode-step kernels (csrc/fused_ops.cu) against fp32 PyTorch references."""
import pytest
import torch

from packmla.formats import codec
from packmla.ops import fused, kv as kv_ops

pytestmark = pytest.mark.gpu

dev = "cuda"


def _ref_norm(x, w, eps):
    return (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w)


@pytest.mark.parametrize("n", [4096, 1024, 512, 130])
@pytest.mark.parametrize("addends", ["none", "bf16", "both"])
def test_add_rmsnorm(n, addends):
    g = torch.Generator(device=dev).manual_seed(n)
    rows = 37
    base = torch.randn(rows, n + 64, device=dev, generator=g).bfloat16()
    x = base[:, :n]  # strided input
    w = torch.rand(n, device=dev, generator=g) + 0.5
    d = torch.randn(rows, n, device=dev, generator=g).bfloat16() if addends != "none" else None
    df = torch.randn(rows, n, device=dev, generator=g) if addends == "both" else None
    x_ref = x.float()
    if d is not None:
        x_ref = x_ref + d.float()
    if df is not None:
        x_ref = x_ref + df
    if addends != "none":
        x_ref = x_ref.bfloat16().float()
    xn, h = fused.add_rmsnorm(x, w, 1e-6, d, df)
    assert torch.equal(xn.float(), x_ref)
    ref = _ref_norm(x_ref, w, 1e-6)
    torch.testing.assert_close(h.float(), ref, atol=2e-2, rtol=1e-2)
    # in place on the residual stream
    xc = x.contiguous().clone()
    xn2, h2 = fused.add_rmsnorm(xc, w, 1e-6, d, df, inplace=True)
    assert torch.equal(h2, h)
    if addends != "none":
        assert xn2.data_ptr() == xc.data_ptr() and torch.equal(xc.float(), x_ref)


def test_rope_q_matches_cpu():
    freqs = kv_ops.freq_table_f32(codec.rope_table(4096, 10000.0))
    g = torch.Generator().manual_seed(1)
    q = torch.randn(5, 16, 512, generator=g).bfloat16()
    pos = torch.tensor([0, 3, 100, 4095, 17])
    ref = fused.rope_q(q.clone(), pos, freqs)
    out = fused.rope_q(q.to(dev), pos.to(dev), freqs.to(dev))
    assert torch.equal(out.cpu(), ref)


@pytest.mark.parametrize("ratio,D", [(4, 512), (128, 512), (4, 128)])
def test_comp_pool_sequence(ratio, D):
    g = torch.Generator().manual_seed(ratio + D)
    slots, B, steps = 6, 3, 2 * ratio + 3
    ape = 0.1 * torch.randn(ratio, D, generator=g)
    st_c = torch.stack((torch.full((slots, D), float("-inf")), torch.zeros(slots, D), torch.zeros(slots, D)), 1)
    st_g = st_c.clone().to(dev)
    req = torch.tensor([4, 0, 2])
    start = torch.tensor([0, 5, ratio - 1])
    for t in range(steps):
        proj = torch.randn(B, 64 + 2 * D, generator=g).bfloat16()
        pos = start + t
        raw_c = fused.comp_pool(proj, 64, D, ape, st_c, req, pos)
        raw_g = fused.comp_pool(proj.to(dev), 64, D, ape.to(dev), st_g, req.to(dev), pos.to(dev))
        torch.testing.assert_close(raw_g.cpu(), raw_c, atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(st_g.cpu(), st_c, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("E,k", [(256, 8), (64, 6), (16, 2)])
def test_route_topk(E, k):
    g = torch.Generator().manual_seed(E)
    T = 50
    logits = (2 * torch.randn(T, E + 8, generator=g)).bfloat16()[:, 8:]
    bias = 0.05 * torch.randn(E, generator=g)
    ids_c, w_c = fused.route_topk(logits, bias, k, 2.5)
    ids_g, w_g = fused.route_topk(logits.to(dev), bias.to(dev), k, 2.5)
    assert torch.equal(ids_g.cpu().long(), ids_c.long())
    torch.testing.assert_close(w_g.cpu(), w_c, atol=1e-6, rtol=1e-5)


def test_silu_mul():
    g = torch.Generator().manual_seed(3)
    gu = torch.randn(9, 2 * 384 + 16, generator=g).bfloat16()[:, :768]
    ref = fused.silu_mul(gu)
    out = fused.silu_mul(gu.to(dev))
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=1e-2, rtol=1e-2)

"""Layout self-tests of the block-scaled tcgen05 path (csrc/bs_probe.cu) that the MXFP4 x MXFP8 MoE
kernel is built on: unpacked FP4 operands, UE8M0 scale factors in TMEM, TMA unpacking loads and
tcgen05.cp scale-factor copies.  Each check is exact (products of FP4, E4M3 and powers of two)."""
import pytest
import torch

from packmla.ops._ext import error_word, ext

pytestmark = pytest.mark.gpu
dev = "cuda"
E2M1 = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6])


def _swizzle(rows: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(rows)
    for r in range(rows.shape[0]):
        for u in range(8):
            v = u ^ (r % 8)
            out[r, 16 * v:16 * v + 16] = rows[r, 16 * u:16 * u + 16]
    return out


def _e4m3(x):
    return x.to(torch.float8_e4m3fn).view(torch.uint8)


def _word(b0, b1=None, b2=None, b3=None):
    b1 = b0 if b1 is None else b1
    b2 = b0 if b2 is None else b2
    b3 = b0 if b3 is None else b3
    w = (b0 & 0xFF) | ((b1 & 0xFF) << 8) | ((b2 & 0xFF) << 16) | ((b3 & 0xFF) << 24)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def _idesc(N, af, bf, asf=0, bsf=0):
    return (bsf << 4) | (af << 7) | (bf << 10) | ((N >> 3) << 17) | (1 << 23) | ((128 >> 4) << 24) | (asf << 29)


def _run(a_rows, b_rows, sfa, sfb, desc, kind):
    err = error_word(torch.device(dev))
    err.zero_()
    d = ext().bs_probe(_swizzle(a_rows).to(dev), _swizzle(b_rows).to(dev), sfa.to(dev).contiguous(),
                       sfb.to(dev).contiguous(), desc, kind, 0, 0, err)
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    return d.cpu()


def test_fp4_operand_is_unpacked_low_half():
    """E2M1 in kind::f8f6f4: 16 values packed in bytes 0-7 of each 16-byte chunk (low nibble first)."""
    codes = torch.tensor([[(m * 3 + k) % 16 for k in range(32)] for m in range(128)], dtype=torch.uint8)
    a = torch.zeros(128, 128, dtype=torch.uint8)
    for c in range(2):
        el = codes[:, 16 * c:16 * c + 16]
        a[:, 16 * c:16 * c + 8] = el[:, 0::2] | (el[:, 1::2] << 4)
    b = torch.zeros(32, 128, dtype=torch.uint8)
    b[:, :32] = _e4m3(torch.eye(32))
    desc = (1 << 4) | (5 << 7) | ((32 >> 3) << 17) | ((128 >> 4) << 24)
    d = _run(a, b, torch.zeros(128, 16, dtype=torch.int32), torch.zeros(128, 16, dtype=torch.int32), desc, 0)
    assert torch.equal(d, E2M1[codes.long()])


@pytest.mark.parametrize("N", [8, 16, 64, 256])
def test_scale_factor_tmem_layout(N):
    """Row m of A reads lane m, column m / 32; column n of B reads lane 32 q + n % 32, column n / 32."""
    ones_a = torch.zeros(128, 128, dtype=torch.uint8)
    ones_a[:, :32] = _e4m3(torch.ones(128, 32))
    ones_b = torch.zeros(N, 128, dtype=torch.uint8)
    ones_b[:, :32] = _e4m3(torch.ones(N, 32))
    lane = torch.arange(128)[:, None].expand(128, 16)
    col = torch.arange(16)[None].expand(128, 16)
    # distinct exponents per (lane, column) for A, per (lane % 32, column) for B
    sfa = _word(127 + (lane % 32) - 16 + 3 * col)
    sfb = _word(127 + (lane % 32) - 16 - 2 * col)
    d = _run(ones_a, ones_b, sfa, sfb, _idesc(N, 0, 0), 1)
    m = torch.arange(128)[:, None].float()
    n = torch.arange(N)[None].float()
    ea = (m % 32) - 16 + 3 * torch.floor(m / 32)
    eb = (n % 32) - 16 - 2 * torch.floor(n / 32)
    assert torch.equal(d, 32 * torch.exp2(ea + eb))


def test_scale_factor_byte_select():
    ones_a = torch.zeros(128, 128, dtype=torch.uint8)
    ones_a[:, :32] = _e4m3(torch.ones(128, 32))
    ones_b = torch.zeros(16, 128, dtype=torch.uint8)
    ones_b[:, :32] = _e4m3(torch.ones(16, 32))
    t = torch.zeros(128, 16, dtype=torch.int64)
    sfa = _word(t + 124, t + 128, t + 132, t + 136)
    sfb = _word(t + 127, t + 126, t + 125, t + 124)
    for sid in range(4):
        d = _run(ones_a, ones_b, sfa, sfb, _idesc(16, 0, 0, sid, sid), 1)
        assert torch.all(d == 32 * 2.0 ** ((4 * sid - 3) - sid))


@pytest.mark.parametrize("k_steps", [1, 4])
def test_tma_unpack_and_tmem_cp_pipeline(k_steps):
    g = torch.Generator().manual_seed(k_steps)
    codes = torch.randint(0, 16, (128, 128), generator=g, dtype=torch.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    img = torch.zeros(128, 128, dtype=torch.uint8)
    for c in range(8):
        img[:, 16 * c:16 * c + 8] = packed[:, 8 * c:8 * c + 8]
    N = 16
    bv = torch.randint(-8, 9, (N, 128), generator=g).float() / 4
    sfa = torch.randint(124, 131, (128, 4), generator=g, dtype=torch.uint8)
    sfb = torch.randint(124, 131, (N, 4), generator=g, dtype=torch.uint8)
    sfa_src = torch.zeros(32, 16, dtype=torch.uint8)
    for q in range(4):
        sfa_src[:, 4 * q:4 * q + 4] = sfa[32 * q:32 * q + 32]
    sfb_src = torch.zeros(32, 16, dtype=torch.uint8)
    sfb_src[:N, :4] = sfb
    err = error_word(torch.device(dev))
    err.zero_()
    d, dump = ext().bs_probe2(packed.to(dev), _swizzle(_e4m3(bv)).to(dev), sfa_src.to(dev), sfb_src.to(dev),
                              k_steps, 8192, err)
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    # TMA writes the data half of each 16-byte chunk; the padding half keeps whatever was there
    data = torch.zeros(128, 128, dtype=torch.bool)
    for c in range(8):
        data[:, 16 * c:16 * c + 8] = True
    data = _swizzle(data.to(torch.uint8)).bool()
    assert torch.equal(dump.cpu()[data], _swizzle(img)[data])
    K = 32 * k_steps
    sa = torch.exp2(sfa.float() - 127).repeat_interleave(32, 1)[:, :K]
    sb = torch.exp2(sfb.float() - 127).repeat_interleave(32, 1)[:, :K]
    ref = (E2M1[codes.long()][:, :K] * sa) @ (bv[:, :K] * sb).T
    assert torch.equal(d.cpu(), ref)

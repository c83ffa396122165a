"""GPU: the sparse-MLA decode kernel writes only its own output rows.

`out` and `lse` are given as leading views of larger buffers whose trailing rows hold a canary value
(-91); after the call the canaries must be intact, and the viewed rows must equal a call that
allocated its own outputs (within the tolerance of the other decode tests).
"""
import pytest
import torch
from test_gpu_kernels import _build_cache

from packmla.ops import attention as attn_ops
from packmla.ops import check_errors

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("packed", [False, True])
def test_decode_outputs_leave_canary_rows_intact(cuda, packed):
    B, H, K, W = 3, 64, 317, 128
    g = torch.Generator().manual_seed(91 + int(packed))
    n_swa, n_csa = 2 * W * B, 4 * K * B
    freqs, swa_pool, csa_pool, planes, posrow = _build_cache(91, n_swa, n_csa, packed)
    csa_slots = torch.randint(0, n_csa, (B, K), generator=g, dtype=torch.int32)
    args = dict(swa_slots=torch.randint(0, n_swa, (B, W), generator=g, dtype=torch.int32),
                swa_len=torch.full((B,), W, dtype=torch.int32), csa_slots=csa_slots,
                csa_pos=posrow[csa_slots.long()].int(), csa_len=torch.tensor([K, K // 2, 1], dtype=torch.int32),
                sink=torch.randn(H, generator=g), q_pos=torch.randint(0, 8000, (B,), generator=g, dtype=torch.int32))
    dev = {k: v.cuda() for k, v in args.items()}
    q = (torch.randn(B, H, 512, generator=g) / 2).bfloat16().cuda()
    gplanes = None if planes is None else attn_ops.PackedPlanes(planes.values.cuda(), planes.bitmap.cuda(),
                                                                planes.scales.cuda())
    common = dict(freqs=freqs.cuda(), scale=512 ** -0.5, csa_pool=None if csa_pool is None else csa_pool.cuda(),
                  csa_planes=gplanes, **dev)
    ref_o, ref_l = attn_ops.sparse_mla_decode(q, swa_pool.cuda(), **common)
    out_big = torch.full((B + 2, H, 512), -91.0, dtype=torch.bfloat16, device=cuda)
    lse_big = torch.full((B + 2, H), -91.0, dtype=torch.float32, device=cuda)
    o, lse = attn_ops.sparse_mla_decode(q, swa_pool.cuda(), out=out_big[:B], lse=lse_big[:B], **common)
    torch.cuda.synchronize()
    check_errors(cuda)
    assert o.data_ptr() == out_big.data_ptr() and lse.data_ptr() == lse_big.data_ptr()
    assert bool((out_big[B:] == -91.0).all()) and bool((lse_big[B:] == -91.0).all())
    torch.testing.assert_close(out_big[:B].float(), ref_o.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse_big[:B], ref_l, atol=2e-2, rtol=2e-2)

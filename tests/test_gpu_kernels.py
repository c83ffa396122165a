"""GPU numerics of the sm_100a kernels against the fp32 CPU oracle."""
import pytest
import torch

from packmla.formats import abi, codec
from packmla.ops import check_errors, ext
from packmla.ops import attention as attn_ops
from packmla.ops import kv as kv_ops

pytestmark = pytest.mark.gpu


def _freqs(n=1 << 14):
    return kv_ops.freq_table_f32(codec.rope_table(n))


@pytest.mark.parametrize("rows", [1, 7, 24, 300])
def test_native_store_byte_exact(cuda, rows):
    g = torch.Generator().manual_seed(rows)
    raw = torch.randn(rows, 512, generator=g) * 3
    raw[0, :7] = 0.0
    weight = torch.rand(512, generator=g) + 0.25
    freqs = _freqs()
    pos = torch.randint(0, 4000, (rows,), generator=g)
    pages = (rows + 63) // 64 + 1
    slots = torch.randperm(pages * 64, generator=g)[:rows]
    slots[rows // 2] = -1  # invalid destination writes nothing
    pool = torch.full((pages * abi.NATIVE_PAGE_BYTES,), 0xA5, dtype=torch.uint8)
    gpool = pool.cuda()
    kv_ops.native_store(raw.cuda(), weight.cuda(), 1e-6, slots.cuda(), pos.cuda(), freqs.cuda(), gpool)
    check_errors(cuda)
    kv_ops.native_store(raw, weight, 1e-6, slots, pos, freqs, pool)
    assert torch.equal(gpool.cpu(), pool)


@pytest.mark.parametrize("rows", [1, 24, 257])
def test_packed_store_byte_exact_and_ties(cuda, rows):
    g = torch.Generator().manual_seed(100 + rows)
    raw = torch.randn(rows, 512, generator=g)
    raw[0] = torch.round(raw[0] * 2) / 2  # many exact magnitude ties
    if rows > 1:
        raw[1] = 1.0  # all equal: keep the lowest 256 coordinates
    weight = torch.rand(512, generator=g) + 0.25
    n = rows + 5
    slots = torch.randperm(n, generator=g)[:rows]
    values = torch.full((n, 256), 7, dtype=torch.uint8)
    bitmap = torch.zeros((n, 8), dtype=torch.int64)
    scales = torch.zeros((n, 8), dtype=torch.uint8)
    gv, gb, gs = values.cuda(), bitmap.cuda(), scales.cuda()
    kv_ops.packed_store(raw.cuda(), weight.cuda(), 1e-6, slots.cuda(), gv, gb, gs)
    check_errors(cuda)
    kv_ops.packed_store(raw, weight, 1e-6, slots, values, bitmap, scales)
    assert torch.equal(gb.cpu(), bitmap)
    assert torch.equal(gs.cpu(), scales)
    assert torch.equal(gv.cpu(), values)


@pytest.mark.parametrize("mode,K,N", [(0, 128, 64), (0, 64, 16), (1, 128, 64), (1, 32, 16), (1, 64, 32),
                                      (2, 128, 16), (2, 64, 64), (2, 32, 32), (3, 128, 64), (3, 64, 16)])
def test_umma_operand_layouts(cuda, mode, K, N):
    g = torch.Generator().manual_seed(K + N + mode)
    err = torch.zeros(4, dtype=torch.int32, device=cuda)
    if mode in (0, 2):
        a = torch.randn(128, K, generator=g).bfloat16()
        b = torch.randn(N, K, generator=g).bfloat16()
        ref = a.float() @ b.float().T
    else:
        a = torch.randn(K, 128, generator=g).bfloat16()
        b = torch.randn(K, N, generator=g).bfloat16()
        ref = a.float().T @ b.float()
    if mode == 3:  # E4M3 codes
        a8 = (torch.randn(128, K, generator=g) * 4).to(torch.float8_e4m3fn)
        b8 = (torch.randn(N, K, generator=g) * 4).to(torch.float8_e4m3fn)
        a, b = a8.view(torch.uint8), b8.view(torch.uint8)
        ref = a8.float() @ b8.float().T
    d = ext().umma_probe(a.cuda(), b.cuda(), mode, err)
    assert err.cpu()[0] == 0
    torch.testing.assert_close(d.cpu(), ref, atol=1e-2, rtol=1e-2)


def _build_cache(seed, n_swa_rows, n_csa_rows, packed):
    g = torch.Generator().manual_seed(seed)
    freqs = _freqs()
    w = torch.rand(512, generator=g) + 0.5
    swa_pages = (n_swa_rows + 63) // 64
    swa_pool = torch.zeros(swa_pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8)
    swa_raw = torch.randn(n_swa_rows, 512, generator=g)
    kv_ops.native_store(swa_raw, w, 1e-6, torch.arange(n_swa_rows), torch.randint(0, 8000, (n_swa_rows,), generator=g),
                        freqs, swa_pool)
    csa_raw = torch.randn(n_csa_rows, 512, generator=g)
    csa_posrow = torch.randint(0, 8000, (n_csa_rows,), generator=g)
    if packed:
        planes = attn_ops.PackedPlanes(torch.zeros(n_csa_rows, 256, dtype=torch.uint8),
                                       torch.zeros(n_csa_rows, 8, dtype=torch.int64),
                                       torch.zeros(n_csa_rows, 8, dtype=torch.uint8))
        kv_ops.packed_store(csa_raw, w, 1e-6, torch.arange(n_csa_rows), planes.values, planes.bitmap, planes.scales)
        return freqs, swa_pool, None, planes, csa_posrow
    pages = (n_csa_rows + 63) // 64
    csa_pool = torch.zeros(pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8)
    kv_ops.native_store(csa_raw, w, 1e-6, torch.arange(n_csa_rows), csa_posrow, freqs, csa_pool)
    return freqs, swa_pool, csa_pool, None, csa_posrow


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("B,H,K,splits,qscale", [(2, 64, 512, None, 0.5), (3, 16, 317, 1, 0.5),
                                                  (2, 128, 512, 3, 0.5), (1, 8, 40, None, 0.5),
                                                  (2, 64, 512, 1, 0.5), (3, 64, 317, 2, 0.5),
                                                  (1, 64, 1536, 1, 0.5), (2, 64, 1024, 1, 24.0),
                                                  (2, 32, 700, 3, 24.0), (2, 32, 700, 4, 24.0),
                                                  (1, 64, 1536, 8, 0.5), (2, 64, 512, 16, 0.5)])
def test_sparse_decode_matches_oracle(cuda, packed, B, H, K, splits, qscale):
    """GPU decode vs the fp32 oracle.  One split runs every 128-row tile of a query in one CTA and writes the
    output; 2, 4 or 8 splits are one thread-block cluster that merges in distributed shared memory (some
    splits with no tile, a head group short of 64); other counts go through the partials and the combine
    kernel; a large query scale makes the per-head maxima grow from tile to tile, so the O rescale runs."""
    seed = B * 1000 + H + K + int(packed)
    g = torch.Generator().manual_seed(seed)
    W = 128
    n_swa, n_csa = 2 * W * B, 4 * K * B
    freqs, swa_pool, csa_pool, planes, posrow = _build_cache(seed, n_swa, n_csa, packed)
    swa_slots = torch.randint(0, n_swa, (B, W), generator=g, dtype=torch.int32)
    swa_len = torch.randint(W // 2, W + 1, (B,), generator=g, dtype=torch.int32)
    csa_slots = torch.randint(0, n_csa, (B, K), generator=g, dtype=torch.int32)
    csa_slots[0, 3] = -1  # masked selection
    csa_len = torch.randint(K // 2, K + 1, (B,), generator=g, dtype=torch.int32)
    csa_len[0] = K
    csa_pos = posrow[csa_slots.clamp(min=0).long()].int()
    q = (torch.randn(B, H, 512, generator=g) * qscale).bfloat16()
    sink = torch.randn(H, generator=g)
    q_pos = torch.randint(0, 8000, (B,), generator=g, dtype=torch.int32)
    scale = 1 / 512 ** 0.5
    args = dict(swa_slots=swa_slots, swa_len=swa_len, csa_slots=csa_slots, csa_pos=csa_pos, csa_len=csa_len,
                sink=sink, scale=scale, q_pos=q_pos)
    ref_o, ref_lse = attn_ops.sparse_mla_decode(q, swa_pool, freqs=freqs, csa_pool=csa_pool, csa_planes=planes, **args)
    dev = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in args.items()}
    gplanes = None if planes is None else attn_ops.PackedPlanes(planes.values.cuda(), planes.bitmap.cuda(),
                                                                planes.scales.cuda())
    o, lse = attn_ops.sparse_mla_decode(q.cuda(), swa_pool.cuda(), freqs=freqs.cuda(),
                                        csa_pool=None if csa_pool is None else csa_pool.cuda(), csa_planes=gplanes,
                                        num_splits=splits, **dev)
    check_errors(cuda)
    torch.testing.assert_close(o.float().cpu(), ref_o.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("rows", [1, 24, 130])
def test_fp4_store_byte_exact(cuda, packed, rows):
    """FP4 C4 records (V4.1 cache) from the device store equal the CPU codec's bytes, ties included."""
    from packmla.formats import fp4

    g = torch.Generator().manual_seed(300 + rows + int(packed))
    raw = torch.randn(rows, 512, generator=g) * 2
    raw[0] = torch.round(raw[0] * 4) / 4  # many equal magnitudes after quantization
    if rows > 1:
        raw[1] = 1.0
    weight = torch.rand(512, generator=g) + 0.25
    freqs = _freqs()
    pos = torch.randint(0, 4000, (rows,), generator=g)
    pages = (rows + 63) // 64 + 1
    slots = torch.randperm(pages * 64, generator=g)[:rows]
    if rows > 2:
        slots[2] = -1
    fmt = "direct" if packed else "native"
    pool = torch.full((pages * fp4.page_bytes(fmt),), 0x5A, dtype=torch.uint8)
    gpool = pool.cuda()
    kv_ops.fp4_store(raw.cuda(), weight.cuda(), 1e-6, slots.cuda(), pos.cuda(), freqs.cuda(), gpool, packed)
    check_errors(cuda)
    kv_ops.fp4_store(raw, weight, 1e-6, slots, pos, freqs, pool, packed)
    assert torch.equal(gpool.cpu(), pool)


@pytest.mark.parametrize("fmt", ["native", "direct"])
@pytest.mark.parametrize("B,H,K,splits,qscale", [(2, 64, 512, None, 0.5), (3, 16, 317, 1, 0.5),
                                                  (2, 128, 512, 3, 0.5), (2, 64, 1024, 2, 24.0),
                                                  (1, 64, 1536, 8, 0.5)])
def test_fp4_decode_matches_oracle(cuda, fmt, B, H, K, splits, qscale):
    """GPU decode over FP4 C4 records (V4.1 cache: Native 288 B / Packed 224 B) beside Native SWA rows vs the
    fp32 oracle, which decodes the same pages on the CPU."""
    from packmla.formats import fp4

    seed = 7000 + B * 100 + H + K
    g = torch.Generator().manual_seed(seed)
    W = 128
    n_swa, n_csa = 2 * W * B, 4 * K * B
    freqs, swa_pool, _, _, posrow = _build_cache(seed, n_swa, 0, False)
    w = torch.rand(512, generator=g) + 0.5
    pages = (n_csa + 63) // 64
    pool = torch.zeros(pages * fp4.page_bytes(fmt), dtype=torch.uint8)
    posrow = torch.randint(0, 8000, (n_csa,), generator=g)
    kv_ops.fp4_store(torch.randn(n_csa, 512, generator=g), w, 1e-6, torch.arange(n_csa), posrow, freqs, pool,
                     fmt == "direct")
    swa_slots = torch.randint(0, n_swa, (B, W), generator=g, dtype=torch.int32)
    swa_len = torch.randint(W // 2, W + 1, (B,), generator=g, dtype=torch.int32)
    csa_slots = torch.randint(0, n_csa, (B, K), generator=g, dtype=torch.int32)
    csa_slots[0, 3] = -1
    csa_len = torch.randint(K // 2, K + 1, (B,), generator=g, dtype=torch.int32)
    csa_len[0] = K
    csa_pos = posrow[csa_slots.clamp(min=0).long()].int()
    q = (torch.randn(B, H, 512, generator=g) * qscale).bfloat16()
    sink = torch.randn(H, generator=g)
    q_pos = torch.randint(0, 8000, (B,), generator=g, dtype=torch.int32)
    args = dict(swa_slots=swa_slots, swa_len=swa_len, csa_slots=csa_slots, csa_pos=csa_pos, csa_len=csa_len,
                sink=sink, scale=1 / 512 ** 0.5, q_pos=q_pos)
    ref_o, ref_lse = attn_ops.sparse_mla_decode(q, swa_pool, freqs=freqs, csa_pool=pool, csa_fp4=fmt, **args)
    dev = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in args.items()}
    o, lse = attn_ops.sparse_mla_decode(q.cuda(), swa_pool.cuda(), freqs=freqs.cuda(), csa_pool=pool.cuda(),
                                        csa_fp4=fmt, num_splits=splits, **dev)
    check_errors(cuda)
    torch.testing.assert_close(o.float().cpu(), ref_o.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=2e-2, rtol=2e-2)

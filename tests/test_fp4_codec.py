"""FP4 C4 record codec (packmla.formats.fp4): E2M1 rounding, per-16 E4M3 scales, Packed survivor
selection, MSB-first bitmap, nibble order and page layout, against direct restatements in fp32."""
import torch

from packmla.formats import abi, codec, fp4


def _rows(n=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, abi.LATENT_DIM, generator=g) * torch.rand(n, 1, generator=g) * 3
    return x.to(torch.bfloat16).float()


def test_record_sizes():
    assert fp4.NATIVE_RECORD_BYTES == 288 and fp4.PACKED_RECORD_BYTES == 224
    assert fp4.record_bytes("native") == 288 and fp4.record_bytes("direct") == 224
    assert abs(1 - 224 / 288 - 0.2222) < 1e-4  # global records shrink 22.22%


def test_e2m1_grid_ties_and_saturation():
    grid = fp4.E2M1_GRID
    assert torch.equal(fp4.e2m1_decode(fp4.e2m1_encode(grid)), grid)
    assert torch.equal(fp4.e2m1_decode(fp4.e2m1_encode(-grid[1:])), -grid[1:])
    # midpoints go to the even code: 0.25->0, 0.75->1.0, 1.25->1.0, 1.75->2, 2.5->2, 3.5->4, 5->4
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    assert fp4.e2m1_decode(fp4.e2m1_encode(mids)).tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0]
    assert fp4.e2m1_decode(fp4.e2m1_encode(torch.tensor([7.0, -100.0]))).tolist() == [6.0, -6.0]
    assert int(fp4.e2m1_encode(torch.tensor([-0.1]))[0]) == 0  # no negative zero code
    # off-midpoint values: nearest grid point by brute force
    x = torch.linspace(-6, 6, 1201)
    ref = grid[(x.abs()[:, None] - grid).abs().argmin(-1)] * x.sign()
    near_mid = ((x.abs()[:, None] - (grid[:-1] + grid[1:]) / 2).abs() < 1e-6).any(-1)
    got = fp4.e2m1_decode(fp4.e2m1_encode(x))
    assert torch.equal(got[~near_mid], ref[~near_mid])


def test_native_roundtrip_within_one_scale_step():
    rows = _rows()
    codes, scales = fp4.native_encode(rows)
    assert codes.shape == (rows.shape[0], 256) and scales.shape == (rows.shape[0], 32)
    dec = fp4.native_decode(codes, scales)
    s = scales.view(torch.float8_e4m3fn).float().repeat_interleave(16, -1)
    # half the widest E2M1 gap (1) plus scale-rounding saturation (< 0.4) in units of the scale
    assert bool(((dec - rows).abs() <= s + 1e-6).all())
    # even coordinates in low nibbles
    c0 = fp4.e2m1_encode(rows[:, 0] / s[:, 0])
    assert torch.equal(codes[:, 0] & 0xF, c0)


def test_scale_is_e4m3_of_group_amax_over_six():
    rows = _rows(3, 1)
    _, scales = fp4.native_encode(rows)
    amax = rows.view(3, 32, 16).abs().amax(-1)
    assert torch.equal(scales, (amax / 6).to(torch.float8_e4m3fn).view(torch.uint8))


def test_packed_keeps_top_dequantized_with_lower_coordinate_ties():
    rows = _rows(4, 2)
    codes, scales = fp4.native_encode(rows)
    native = fp4.native_decode(codes, scales)
    pc, words, ps = fp4.packed_encode(rows)
    assert pc.shape == (4, 128) and words.shape == (4, 8) and torch.equal(ps, scales)
    mask = fp4.mask_from_msb_bitmap(words)
    assert bool((mask.sum(-1) == 256).all())
    for r in range(4):
        mag = native[r].abs()
        kept, dropped = mag[mask[r]], mag[~mask[r]]
        assert float(kept.min()) >= float(dropped.max())
        # among equal magnitudes at the threshold, every kept coordinate precedes every dropped one
        t = float(kept.min())
        idx = torch.arange(512)
        at_t = mag == t
        if bool((at_t & ~mask[r]).any()):
            assert int(idx[at_t & mask[r]].max()) < int(idx[at_t & ~mask[r]].min())
    assert torch.equal(fp4.packed_decode(pc, words, ps), native * mask)


def test_all_equal_row_keeps_first_256_coordinates():
    rows = torch.full((1, 512), 0.5)
    pc, words, ps = fp4.packed_encode(rows)
    mask = fp4.mask_from_msb_bitmap(words)[0]
    assert bool(mask[:256].all()) and not bool(mask[256:].any())
    assert words[0, :4].tolist() == [-1] * 4 and words[0, 4:].tolist() == [0] * 4


def test_bitmap_is_msb_first_and_ranks_pack_low_nibble_first():
    rows = torch.zeros(1, 512)
    keep = list(range(0, 512, 2))  # 256 survivors: every even coordinate
    vals = torch.linspace(1, 6, 256)
    rows[0, keep] = vals
    pc, words, ps = fp4.packed_encode(rows)
    mask = fp4.mask_from_msb_bitmap(words)[0]
    assert mask.nonzero()[:, 0].tolist() == keep
    # coordinate 64w + b is bit 63 - b: even coordinates set bits 63, 61, ..., 1
    expect = sum(1 << (63 - b) for b in range(0, 64, 2))
    expect -= 1 << 64  # two's complement of a word with bit 63 set
    assert words[0].tolist() == [expect] * 8
    native_codes, _ = fp4.native_encode(rows)
    nib = torch.stack((native_codes[0] & 0xF, native_codes[0] >> 4), -1).reshape(-1)
    surv = nib[keep]
    assert torch.equal(pc[0] & 0xF, surv[0::2]) and torch.equal(pc[0] >> 4, surv[1::2])


def test_rotated_rows_apply_rope_then_bf16():
    rows = _rows(2, 3)
    table = codec.rope_table(64)
    freqs = table[torch.tensor([5, 17])]
    y = fp4.rotated_rows(rows, freqs)
    assert torch.equal(y[:, :448], rows[:, :448])
    assert torch.equal(y, codec.rotate_tail(rows, freqs).to(torch.bfloat16).float())


def test_page_layout_data_rows_then_scale_rows():
    rows = _rows(abi.RECORDS_PER_PAGE, 4)
    for fmt, data_row in (("native", 256), ("direct", 192)):
        page = fp4.write_page(fmt, rows)
        assert page.numel() == fp4.page_bytes(fmt) == abi.RECORDS_PER_PAGE * (data_row + 32)
        _, scales = fp4.native_encode(rows)
        assert torch.equal(page[abi.RECORDS_PER_PAGE * data_row:].view(-1, 32), scales)
        back = fp4.read_page(fmt, page)
        if fmt == "native":
            assert torch.equal(back, fp4.native_decode(*fp4.native_encode(rows)))
        else:
            assert torch.equal(back, fp4.packed_decode(*fp4.packed_encode(rows)))


def test_huge_groups_saturate_the_scale():
    rows = torch.zeros(1, 512)
    rows[0, :16] = 1e6
    codes, scales = fp4.native_encode(rows)
    assert scales[0, 0].view(torch.float8_e4m3fn).float().item() == 448.0
    assert bool(torch.isfinite(fp4.native_decode(codes, scales)).all())


def test_fp4_sparse_decode_reference_matches_dense_attention():
    from packmla.oracle.attention import sparse_mla_decode

    g = torch.Generator().manual_seed(5)
    n_pages, R = 3, abi.RECORDS_PER_PAGE
    for fmt in ("native", "direct"):
        rows = _rows(n_pages * R, 6)
        pool = torch.stack([fp4.write_page(fmt, rows[p * R:(p + 1) * R]) for p in range(n_pages)])
        B, H, K = 2, 4, 20
        idx = torch.randint(0, n_pages * R, (B, K), generator=g)
        idx[0, 3] = -1
        lens = torch.tensor([K, 13])
        swa = [torch.randn(5, 512, generator=g).bfloat16().float() for _ in range(B)]
        q = torch.randn(B, H, 512, generator=g)
        sink, freqs = torch.randn(H, generator=g), codec.rope_table(16)[torch.tensor([3, 9])]
        out, lse = fp4.sparse_decode_reference(q, pool, fmt, idx, lens, swa, sink, 512 ** -0.5, freqs)
        decoded = fp4.native_decode(*fp4.native_encode(rows)) if fmt == "native" else \
            fp4.packed_decode(*fp4.packed_encode(rows))
        kv = []
        for b in range(B):
            sel = idx[b, :int(lens[b])]
            kv.append(torch.cat((swa[b], decoded[sel[sel >= 0]])))
        ref_o, ref_l = sparse_mla_decode(q, kv, sink, 512 ** -0.5, freqs)
        assert torch.equal(out, ref_o) and torch.equal(lse, ref_l)
        assert kv[0].shape[0] == 5 + K - 1 and kv[1].shape[0] == 5 + 13


def test_fp4_capacity_gain_is_below_the_record_shrink():
    from packmla.config import ModelConfig

    cfg = ModelConfig()
    native = fp4.capacity_tokens(cfg, "native", 1 << 30)
    direct = fp4.capacity_tokens(cfg, "direct", 1 << 30)
    gain = direct / native
    assert 1.0 < gain < 288 / 224  # indexer keys, C128 records and the SWA share do not shrink


def test_fp4_store_cpu_path_writes_the_page_layout():
    """The op's CPU path, filling one page through a slot permutation, writes write_page's bytes."""
    from packmla.formats import codec, fp4
    from packmla.ops import kv as kv_ops

    g = torch.Generator().manual_seed(5)
    raw = torch.randn(64, 512, generator=g)
    w = torch.rand(512, generator=g) + 0.5
    freqs = kv_ops.freq_table_f32(codec.rope_table(128))
    pos = torch.randint(0, 128, (64,), generator=g)
    slots = torch.randperm(64, generator=g)
    rows = fp4.rotated_rows(codec.rms_normalize(raw, w, 1e-6), torch.view_as_complex(freqs[pos].contiguous()))
    order = torch.argsort(slots)
    for packed, fmt in ((False, "native"), (True, "direct")):
        pool = torch.zeros(fp4.page_bytes(fmt), dtype=torch.uint8)
        kv_ops.fp4_store(raw, w, 1e-6, slots, pos, freqs, pool, packed)
        assert torch.equal(pool, fp4.write_page(fmt, rows[order]))


def test_decode_op_cpu_path_matches_the_fp4_reference():
    """The attention op's CPU path over an FP4 pool equals fp4.sparse_decode_reference (SWA rows decoded
    from their Native pool)."""
    from packmla.formats import abi, codec, fp4
    from packmla.ops import attention as attn_ops
    from packmla.ops import kv as kv_ops

    g = torch.Generator().manual_seed(11)
    freqs = kv_ops.freq_table_f32(codec.rope_table(256))
    w = torch.rand(512, generator=g) + 0.5
    swa_pool = torch.zeros(abi.NATIVE_PAGE_BYTES, dtype=torch.uint8)
    kv_ops.native_store(torch.randn(64, 512, generator=g), w, 1e-6, torch.arange(64), torch.arange(64), freqs, swa_pool)
    for fmt in ("native", "direct"):
        pool = torch.zeros(2 * fp4.page_bytes(fmt), dtype=torch.uint8)
        kv_ops.fp4_store(torch.randn(100, 512, generator=g), w, 1e-6, torch.arange(100), torch.arange(100), freqs,
                         pool, fmt == "direct")
        B, H = 2, 4
        q = torch.randn(B, H, 512, generator=g).bfloat16()
        swa_slots = torch.randint(0, 64, (B, 8), generator=g, dtype=torch.int32)
        swa_len = torch.tensor([8, 5], dtype=torch.int32)
        csa_slots = torch.randint(0, 100, (B, 16), generator=g, dtype=torch.int32)
        csa_slots[1, 2] = -1
        csa_len = torch.tensor([16, 11], dtype=torch.int32)
        sink, q_pos = torch.randn(H, generator=g), torch.tensor([3, 200], dtype=torch.int32)
        o, lse = attn_ops.sparse_mla_decode(q, swa_pool, swa_slots, swa_len, csa_slots, torch.zeros_like(csa_slots),
                                            csa_len, freqs, sink, 0.05, q_pos, csa_pool=pool, csa_fp4=fmt)
        swa_rows = [codec.native_decode(attn_ops.native_pool_read(swa_pool, swa_slots[b, : swa_len[b]].long()))
                    for b in range(B)]
        qf = torch.view_as_complex(freqs[q_pos.long()].contiguous())
        ro, rl = fp4.sparse_decode_reference(q.float(), pool.view(2, -1), fmt, csa_slots, csa_len, swa_rows, sink,
                                             0.05, qf)
        torch.testing.assert_close(o.float(), ro.float(), atol=0, rtol=0)
        torch.testing.assert_close(lse, rl, atol=0, rtol=0)

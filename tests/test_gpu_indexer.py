"""GPU: FP8 indexer kernels (key store, tcgen05 logits, radix top-k) against the CPU oracle."""
import pytest
import torch

from packmla.ops import check_errors, ext
from packmla.ops import indexer as idx_ops

pytestmark = pytest.mark.gpu


def test_index_key_store_byte_exact(cuda):
    g = torch.Generator().manual_seed(0)
    n = 300
    kraw = torch.randn(n, 128, generator=g) * 3
    kraw[5] = 0.0
    slots = torch.randperm(n + 20, generator=g)[:n]
    slots[7] = -1
    keys = torch.zeros(n + 21, 128, dtype=torch.uint8)
    scales = torch.zeros(n + 21)
    gk, gs = keys.cuda(), scales.cuda()
    idx_ops.index_key_store(kraw.cuda(), slots.cuda(), gk, gs)
    check_errors(cuda)
    idx_ops.index_key_store(kraw, slots, keys, scales)
    assert torch.equal(gk.cpu(), keys) and torch.equal(gs.cpu(), scales)


@pytest.mark.parametrize("B,H,R,topk,pages", [(3, 64, 1000, 512, 24), (2, 8, 300, 32, 8), (5, 64, 40, 512, 4)])
def test_index_select_matches_oracle(cuda, B, H, R, topk, pages):
    g = torch.Generator().manual_seed(B * 100 + R)
    rows = pages * B * 64 + 1
    keys = torch.zeros(rows, 128, dtype=torch.uint8)
    scales = torch.ones(rows)
    idx_ops.index_key_store(torch.randn(rows - 1, 128, generator=g), torch.arange(rows - 1), keys, scales)
    # each query owns shuffled whole pages
    perm = torch.randperm(pages * B, generator=g).view(B, pages)
    r = torch.arange(pages * 64)
    phys = (perm[:, r // 64] * 64 + r % 64).int()
    phys[:, R:] = -1
    count = torch.randint(R // 2, R + 1, (B,), generator=g, dtype=torch.int64)
    q = torch.randn(B, H, 128, generator=g).bfloat16()
    w = torch.rand(B, H, generator=g)
    ref_s, ref_p = idx_ops.index_select(q, w, keys, scales, phys, count, R, topk)
    s, p = idx_ops.index_select(q.cuda(), w.cuda(), keys.cuda(), scales.cuda(), phys.cuda().contiguous(),
                                count.cuda(), R, topk)
    check_errors(cuda)
    s, p = s.cpu(), p.cpu()
    for b in range(B):
        n_valid = min(topk, int(count[b]))
        assert int((s[b] >= 0).sum()) == n_valid
        got = set(s[b][s[b] >= 0].tolist())
        want = set(ref_s[b][ref_s[b] >= 0].tolist())
        assert len(got & want) >= 0.98 * len(want)
        # ascending record order and RoPE rows = 4 * record
        rec = p[b][: n_valid] // 4
        assert torch.all(rec[1:] > rec[:-1])
        assert torch.equal(s[b][:n_valid], phys[b][rec.long()])


@pytest.mark.parametrize("B,H", [(7, 64), (2, 64), (9, 16)])
def test_index_select_shared_rows_matches_oracle(cuda, B, H):
    """Queries sharing one physical-row list (a prefill chunk of one request, passed with row stride 0) are
    scored up to four per CTA from the same key tiles; causal counts differ per query.  The logits must
    equal the one-query-per-CTA path's bit for bit, and the selection the CPU oracle's."""
    g = torch.Generator().manual_seed(B * 10 + H)
    pages, R, topk = 24, 1400, 512
    rows = pages * 64 + 1
    keys = torch.zeros(rows, 128, dtype=torch.uint8)
    scales = torch.ones(rows)
    idx_ops.index_key_store(torch.randn(rows - 1, 128, generator=g), torch.arange(rows - 1), keys, scales)
    r = torch.arange(pages * 64)
    row = (torch.randperm(pages, generator=g)[r // 64] * 64 + r % 64).int()
    row[R:] = -1
    count = (R - 5 * B + 5 * torch.arange(B)).to(torch.int64)  # causal: later queries see more records
    q = torch.randn(B, H, 128, generator=g).bfloat16()
    w = torch.rand(B, H, generator=g)
    shared = row.cuda()[None].expand(B, -1)
    dev_args = (q.cuda(), w.cuda(), keys.cuda(), scales.cuda())
    s1, p1 = idx_ops.index_select(*dev_args, shared, count.cuda(), R, topk)
    s2, p2 = idx_ops.index_select(*dev_args, shared.contiguous(), count.cuda(), R, topk)
    check_errors(cuda)
    assert torch.equal(s1, s2) and torch.equal(p1, p2)
    ref_s, _ = idx_ops.index_select(q, w, keys, scales, row[None].expand(B, -1), count, R, topk)
    for b in range(B):
        got = set(s1[b][s1[b] >= 0].tolist())
        want = set(ref_s[b][ref_s[b] >= 0].tolist())
        assert len(got) == min(topk, int(count[b])) and len(got & want) >= 0.98 * len(want)

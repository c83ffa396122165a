"""GPU: GLM-5.3 MLA rows (Native 512 B / Packed 320 B) through the sm_100a store, Adapter and tcgen05 decode,
against the fp32 CPU oracle."""
import pytest
import torch

from packmla.formats import glm
from packmla.ops import check_errors
from packmla.ops.glm import GLMPlanes, glm_packed_to_native, glm_sparse_decode, glm_store

pytestmark = pytest.mark.gpu


def _cache(seed, rows, device):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(rows, 512, generator=g)
    raw[1] = 0.25
    raw[1, 100:400] = 1.0  # ties at the selection threshold: the lower coordinates win
    w = torch.rand(512, generator=g) + 0.5
    pool = torch.zeros(rows, 512, dtype=torch.uint8, device=device)
    planes = GLMPlanes(torch.zeros(rows, 256, dtype=torch.uint8, device=device),
                       torch.zeros(rows, 8, dtype=torch.int64, device=device))
    slots = torch.randperm(rows, generator=g)
    slots[3] = -1
    glm_store(raw.to(device), w.to(device), 1e-6, slots.to(device), pool=pool)
    glm_store(raw.to(device), w.to(device), 1e-6, slots.to(device), planes=planes)
    return raw, w, slots, pool, planes


def test_store_and_adapter_bytes_match_the_oracle(cuda):
    raw, w, slots, pool, planes = _cache(11, 777, cuda)
    check_errors(cuda)
    keep = slots >= 0
    assert torch.equal(pool.cpu()[slots[keep]], glm.native_encode(raw[keep], w, 1e-6))
    v, b = glm.packed_encode(raw[keep], w, 1e-6)
    assert torch.equal(planes.values.cpu()[slots[keep]], v)
    assert torch.equal(planes.bitmap.cpu()[slots[keep]], b)
    rows = torch.tensor([int(slots[0]), -1, int(slots[1]), 776], device=cuda)
    nat = glm_packed_to_native(planes, rows)
    check_errors(cuda)
    ref = glm_packed_to_native(GLMPlanes(planes.values.cpu(), planes.bitmap.cpu()), rows.cpu())
    assert torch.equal(nat.cpu(), ref)


@pytest.mark.parametrize("B,H,K,splits", [(1, 16, 2051, None), (8, 16, 2048, None), (4, 64, 1024, 1),
                                          (3, 16, 700, 4)])
def test_decode_matches_oracle_and_direct_equals_adapter(cuda, B, H, K, splits):
    rows = 4096
    _, _, _, pool, planes = _cache(100 + B + K, rows, cuda)
    g = torch.Generator().manual_seed(B * 1000 + K)
    q = torch.randn(B, H, 512, generator=g).bfloat16()
    sl = torch.randint(0, rows, (B, K), generator=g, dtype=torch.int32)
    sl[0, 5] = -1
    lens = torch.randint(K // 2, K + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = K
    cpu_pool, cpu_planes = pool.cpu(), GLMPlanes(planes.values.cpu(), planes.bitmap.cpu())
    outs = {}
    for name, kw, ckw in (("native", {"pool": pool}, {"pool": cpu_pool}),
                          ("direct", {"planes": planes}, {"planes": cpu_planes})):
        o, lse = glm_sparse_decode(q.to(cuda), sl.to(cuda), lens.to(cuda), num_splits=splits, **kw)
        check_errors(cuda)
        ref_o, ref_lse = glm_sparse_decode(q, sl, lens, **ckw)
        torch.testing.assert_close(o.float().cpu(), ref_o.float(), atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(lse.cpu(), ref_lse, atol=2e-2, rtol=2e-2)
        outs[name] = (o, lse)
    # Direct expands the survivors into the same FP16 K tile the Adapter's Native rows give: equal bits
    flat = sl.clamp(min=0).reshape(-1).long().to(cuda)
    adapted = glm_packed_to_native(planes, flat).view(B * K, 512)
    remap = torch.arange(B * K, dtype=torch.int32, device=cuda).view(B, K)
    remap[sl.to(cuda) < 0] = -1
    o, lse = glm_sparse_decode(q.to(cuda), remap, lens.to(cuda), num_splits=splits, pool=adapted)
    check_errors(cuda)
    assert torch.equal(o, outs["direct"][0]) and torch.equal(lse, outs["direct"][1])


def test_decode_graph_replay(cuda):
    rows, B, H, K = 2048, 4, 16, 2048
    _, _, _, _, planes = _cache(5, rows, cuda)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(B, H, 512, generator=g).bfloat16().to(cuda)
    sl = torch.randint(0, rows, (B, K), generator=g, dtype=torch.int32).to(cuda)
    lens = torch.full((B,), K, dtype=torch.int32, device=cuda)
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device=cuda)
    lse = torch.empty(B, H, dtype=torch.float32, device=cuda)
    from packmla.ops.attention import DecodeWorkspace, choose_splits

    ws = DecodeWorkspace(B, H, choose_splits(B, H, K), cuda)
    glm_sparse_decode(q, sl, lens, planes=planes, out=out, lse=lse, workspace=ws)
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        glm_sparse_decode(q, sl, lens, planes=planes, out=out, lse=lse, workspace=ws)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    check_errors(cuda)
    assert torch.equal(out, eager)


def test_decode_graph_replay_with_changed_inputs_and_canary_rows(cuda):
    """Capture once, then change the planes' rows, the indices and the lengths in place; the replay equals an
    eager call on the new inputs, and rows past the output (canaries) are never written."""
    from packmla.ops.attention import DecodeWorkspace, choose_splits

    rows, B, H, K = 2048, 4, 16, 2048
    _, _, _, _, planes = _cache(7, rows, cuda)
    g = torch.Generator().manual_seed(8)
    q = torch.randn(B, H, 512, generator=g).bfloat16().to(cuda)
    sl = torch.randint(0, rows, (B, K), generator=g, dtype=torch.int32).to(cuda)
    lens = torch.full((B,), K, dtype=torch.int32, device=cuda)
    canary = torch.full((B + 1, H, 512), -91.0, dtype=torch.bfloat16, device=cuda)
    lse_buf = torch.full((B + 1, H), -91.0, dtype=torch.float32, device=cuda)
    out, lse = canary[:B], lse_buf[:B]
    ws = DecodeWorkspace(B, H, choose_splits(B, H, K), cuda)
    glm_sparse_decode(q, sl, lens, planes=planes, out=out, lse=lse, workspace=ws)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        glm_sparse_decode(q, sl, lens, planes=planes, out=out, lse=lse, workspace=ws)
    _, _, _, _, other = _cache(9, rows, cuda)
    planes.values.copy_(other.values)
    planes.bitmap.copy_(other.bitmap)
    sl.copy_(torch.randint(0, rows, (B, K), generator=g, dtype=torch.int32).to(cuda))
    sl[1, 7] = -1
    lens.copy_(torch.tensor([K, 1000, 1, 0], dtype=torch.int32))
    q.copy_(torch.randn(B, H, 512, generator=g).bfloat16())
    graph.replay()
    torch.cuda.synchronize()
    check_errors(cuda)
    ref_o, ref_lse = glm_sparse_decode(q, sl, lens, planes=planes, workspace=ws)
    check_errors(cuda)
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_lse)
    assert bool((canary[B] == -91.0).all()) and bool((lse_buf[B] == -91.0).all())
    cpu_o, _ = glm_sparse_decode(q.cpu(), sl.cpu(), lens.cpu(),
                                 planes=GLMPlanes(planes.values.cpu(), planes.bitmap.cpu()))
    torch.testing.assert_close(out.float().cpu(), cpu_o.float(), atol=2e-2, rtol=2e-2)

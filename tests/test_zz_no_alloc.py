"""GPU: the allocation-free decode entry point, called through its exported C symbol.

Some callers of this library cannot allocate GPU memory where they run attention (a host
runtime that reserved all device memory for its own allocator, or a plugin interface that
only passes input and output buffers).  `packmla_sparse_mla_decode_noalloc` serves them with
a scratch array built into the library.  These tests check it bit for bit against the regular
entry point, which takes caller-allocated scratch, on two calls in a row after a larger call has
filled the scratch; against the fp32 PyTorch reference; at exactly the scratch limit; and that
oversized or misaligned requests are refused on the host.  This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


class NoallocArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("q_stride_b", ctypes.c_int64), ("q_stride_h", ctypes.c_int64),
        ("B", ctypes.c_int32), ("H", ctypes.c_int32),
        ("swa_pool", ctypes.c_void_p), ("swa_pool_bytes", ctypes.c_int64), ("swa_slots", ctypes.c_void_p),
        ("swa_cap", ctypes.c_int32), ("swa_len", ctypes.c_void_p),
        ("csa_packed", ctypes.c_int32), ("csa_pool", ctypes.c_void_p), ("csa_pool_bytes", ctypes.c_int64),
        ("csa_values", ctypes.c_void_p), ("csa_bitmap", ctypes.c_void_p), ("csa_scales", ctypes.c_void_p),
        ("csa_rows", ctypes.c_int64), ("csa_slots", ctypes.c_void_p), ("csa_pos", ctypes.c_void_p),
        ("csa_cap", ctypes.c_int32), ("csa_len", ctypes.c_void_p),
        ("freqs", ctypes.c_void_p), ("freq_rows", ctypes.c_int64), ("sink", ctypes.c_void_p),
        ("scale", ctypes.c_float), ("q_pos", ctypes.c_void_p), ("num_splits", ctypes.c_int32),
        ("out", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("err", ctypes.c_void_p),
    ]


def _lib():
    from packmla import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.packmla_sparse_mla_decode_noalloc
    fn.argtypes = [ctypes.POINTER(NoallocArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    lib.packmla_noalloc_last_error.restype = ctypes.c_char_p
    lib.packmla_noalloc_args_size.restype = ctypes.c_size_t
    # the struct above restates csrc/packmla_noalloc.h: its size must match the library's
    assert ctypes.sizeof(NoallocArgs) == lib.packmla_noalloc_args_size()
    return lib


def _case(seed, packed, B=3, H=64, K=256, W=128):
    from packmla.formats import abi, codec
    from packmla.ops import attention as attn_ops
    from packmla.ops import kv as kv_ops

    g = torch.Generator().manual_seed(seed)
    freqs = kv_ops.freq_table_f32(codec.rope_table(8192)).cuda()
    w = (torch.rand(512, generator=g) + 0.5).cuda()
    n_swa, n_csa = 2 * W * B, 4 * K * B
    swa_pool = torch.zeros(((n_swa + 63) // 64) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device="cuda")
    kv_ops.native_store(torch.randn(n_swa, 512, generator=g).cuda(), w, 1e-6, torch.arange(n_swa).cuda(),
                        torch.randint(0, 8000, (n_swa,), generator=g).cuda(), freqs, swa_pool)
    csa_raw = torch.randn(n_csa, 512, generator=g).cuda()
    posrow = torch.randint(0, 8000, (n_csa,), generator=g)
    planes, csa_pool = None, None
    if packed:
        planes = attn_ops.PackedPlanes(torch.zeros(n_csa, 256, dtype=torch.uint8, device="cuda"),
                                       torch.zeros(n_csa, 8, dtype=torch.int64, device="cuda"),
                                       torch.zeros(n_csa, 8, dtype=torch.uint8, device="cuda"))
        kv_ops.packed_store(csa_raw, w, 1e-6, torch.arange(n_csa).cuda(), planes.values, planes.bitmap, planes.scales)
    else:
        csa_pool = torch.zeros(((n_csa + 63) // 64) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device="cuda")
        kv_ops.native_store(csa_raw, w, 1e-6, torch.arange(n_csa).cuda(), posrow.cuda(), freqs, csa_pool)
    csa_slots = torch.randint(0, n_csa, (B, K), generator=g, dtype=torch.int32)
    csa_slots[0, 1] = -1
    return dict(
        q=(torch.randn(B, H, 512, generator=g) / 2).bfloat16().cuda(),
        swa_pool=swa_pool,
        swa_slots=torch.randint(0, n_swa, (B, W), generator=g, dtype=torch.int32).cuda(),
        swa_len=torch.randint(W // 2, W + 1, (B,), generator=g, dtype=torch.int32).cuda(),
        csa_slots=csa_slots.cuda(), csa_pos=posrow[csa_slots.clamp(min=0).long()].int().cuda(),
        csa_len=torch.randint(K // 2, K + 1, (B,), generator=g, dtype=torch.int32).cuda(),
        freqs=freqs, sink=torch.randn(H, generator=g).cuda(), scale=512 ** -0.5,
        q_pos=torch.randint(0, 8000, (B,), generator=g, dtype=torch.int32).cuda(),
        csa_pool=csa_pool, csa_planes=planes)


def _args(c, splits, out, lse, err, q_ptr=None):
    B, H = c["q"].shape[:2]
    packed = c["csa_planes"] is not None
    p = c["csa_planes"]
    return NoallocArgs(
        q=c["q"].data_ptr() if q_ptr is None else q_ptr, q_stride_b=c["q"].stride(0), q_stride_h=c["q"].stride(1),
        B=B, H=H,
        swa_pool=c["swa_pool"].data_ptr(), swa_pool_bytes=c["swa_pool"].numel(), swa_slots=c["swa_slots"].data_ptr(),
        swa_cap=c["swa_slots"].shape[1], swa_len=c["swa_len"].data_ptr(), csa_packed=int(packed),
        csa_pool=0 if packed else c["csa_pool"].data_ptr(), csa_pool_bytes=0 if packed else c["csa_pool"].numel(),
        csa_values=p.values.data_ptr() if packed else 0, csa_bitmap=p.bitmap.data_ptr() if packed else 0,
        csa_scales=p.scales.data_ptr() if packed else 0, csa_rows=p.values.shape[0] if packed else 0,
        csa_slots=c["csa_slots"].data_ptr(), csa_pos=c["csa_pos"].data_ptr(), csa_cap=c["csa_slots"].shape[1],
        csa_len=c["csa_len"].data_ptr(), freqs=c["freqs"].data_ptr(), freq_rows=c["freqs"].shape[0],
        sink=c["sink"].data_ptr(), scale=c["scale"], q_pos=c["q_pos"].data_ptr(), num_splits=splits,
        out=out.data_ptr(), lse=lse.data_ptr(), err=err.data_ptr())


def _call_noalloc(lib, c, splits):
    B, H = c["q"].shape[:2]
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, H, dtype=torch.float32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    a = _args(c, splits, out, lse, err)
    rc = lib.packmla_sparse_mla_decode_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.packmla_noalloc_last_error()
    torch.cuda.synchronize()
    assert err.cpu()[0] == 0
    return out, lse


@pytest.mark.parametrize("packed", [True, False])
def test_noalloc_entry_point_matches_regular_entry_point_twice(cuda, packed):
    """Same kernel, same inputs: the outputs must be bitwise equal to the regular entry point's, on two
    calls in a row, after a larger call has left its partials in the shared scratch."""
    from packmla.ops import attention as attn_ops

    lib = _lib()
    _call_noalloc(lib, _case(10, packed, B=8), 8)  # fills 8 * 8 * 64 partial rows of the scratch first
    for seed, splits in ((11, 2), (12, 3)):  # two calls in a row, different inputs and split counts
        c = _case(seed, packed)
        ref_o, ref_lse = attn_ops.sparse_mla_decode(num_splits=splits, **c)
        out, lse = _call_noalloc(lib, c, splits)
        assert torch.equal(out, ref_o)
        assert torch.equal(lse, ref_lse)


def test_noalloc_entry_point_matches_fp32_oracle(cuda):
    """The allocation-free entry point against the plain PyTorch fp32 reference of the same attention."""
    from packmla.ops import attention as attn_ops

    lib = _lib()
    c = _case(14, True, B=2, K=64, W=32)
    out, lse = _call_noalloc(lib, c, 2)
    cpu = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    if c["csa_planes"] is not None:
        p = c["csa_planes"]
        cpu["csa_planes"] = attn_ops.PackedPlanes(p.values.cpu(), p.bitmap.cpu(), p.scales.cpu())
    ref_o, ref_lse = attn_ops.sparse_mla_decode(**cpu)
    torch.testing.assert_close(out.float().cpu(), ref_o.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse.cpu(), ref_lse.float(), atol=2e-2, rtol=2e-2)


def test_noalloc_accepts_exactly_the_scratch_limit(cuda):
    """B * num_splits * H == 4096 partial rows fills the scratch exactly; the result matches the regular path."""
    from packmla.ops import attention as attn_ops

    lib = _lib()
    assert lib.packmla_noalloc_max_parts() == 4096
    # 16 splits (not a cluster size): every (query, split, head) row of the scratch is written and read
    c = _case(15, True, B=4, H=64, K=128, W=64)
    ref_o, ref_lse = attn_ops.sparse_mla_decode(num_splits=16, **c)
    out, lse = _call_noalloc(lib, c, 16)
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_lse)


def test_noalloc_rejects_oversized_request(cuda):
    lib = _lib()
    # 4097 = 17 * 241 partial rows: one more than the scratch holds; rejected on the host before any launch
    a = NoallocArgs(B=17, H=241, num_splits=1, swa_pool_bytes=0, csa_packed=1)
    rc = lib.packmla_sparse_mla_decode_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"4096" in lib.packmla_noalloc_last_error()


def test_noalloc_rejects_misaligned_q_on_the_host(cuda):
    """A q pointer that is not 16-byte aligned would make the kernel's vector loads fault: it is refused
    before launch, and the same arguments with the aligned pointer then run."""
    lib = _lib()
    c = _case(16, True, B=2, K=64, W=32)
    out = torch.empty(2, 64, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(2, 64, dtype=torch.float32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    bad = _args(c, 1, out, lse, err, q_ptr=c["q"].data_ptr() + 2)
    rc = lib.packmla_sparse_mla_decode_noalloc(ctypes.byref(bad), torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"16-byte" in lib.packmla_noalloc_last_error()
    torch.cuda.synchronize()
    assert err.cpu()[0] == 0
    good = _args(c, 1, out, lse, err)
    assert lib.packmla_sparse_mla_decode_noalloc(ctypes.byref(good), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert err.cpu()[0] == 0

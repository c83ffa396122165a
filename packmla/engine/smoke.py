"""Tiny end-to-end check on one GPU (used by the driver's smoke step)."""
from __future__ import annotations

import torch


def run_smoke(device: torch.device) -> None:
    from ..formats import abi, codec
    from ..ops import attention as attn_ops
    from ..ops import check_errors
    from ..ops import kv as kv_ops

    torch.manual_seed(0)
    freqs = kv_ops.freq_table_f32(codec.rope_table(4096)).to(device)
    w = torch.ones(512, device=device)
    rows = 256
    raw = torch.randn(rows, 512, device=device)
    pool = torch.zeros(4 * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=device)
    kv_ops.native_store(raw, w, 1e-6, torch.arange(rows, device=device), torch.arange(rows, device=device), freqs, pool)
    planes = attn_ops.PackedPlanes(torch.zeros(rows, 256, dtype=torch.uint8, device=device),
                                   torch.zeros(rows, 8, dtype=torch.int64, device=device),
                                   torch.zeros(rows, 8, dtype=torch.uint8, device=device))
    kv_ops.packed_store(raw, w, 1e-6, torch.arange(rows, device=device), planes.values, planes.bitmap, planes.scales)
    B, H = 2, 64
    q = torch.randn(B, H, 512, device=device).bfloat16()
    swa = torch.arange(128, device=device, dtype=torch.int32).repeat(B, 1)
    csa = torch.arange(128, 256, device=device, dtype=torch.int32).repeat(B, 1)
    out, lse = attn_ops.sparse_mla_decode(
        q, pool, swa, torch.full((B,), 128, dtype=torch.int32, device=device), csa, csa * 4,
        torch.full((B,), 128, dtype=torch.int32, device=device), freqs, torch.zeros(H, device=device),
        512 ** -0.5, torch.zeros(B, dtype=torch.int32, device=device), csa_planes=planes)
    torch.cuda.synchronize(device)
    check_errors(device)
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()
    run_model_smoke(device)


def run_model_smoke(device: torch.device) -> None:
    """Prefill + CUDA-graph decode of a small V4-Flash-shape model (MXFP4 experts, Direct KV, HiCache on):
    the store, indexer, attention, fused-op and MoE kernels of the serving step all run once."""
    from ..config import EngineConfig, ModelConfig
    from ..engine.engine import Engine, SamplingParams
    from ..ops import check_errors

    cfg = ModelConfig(name="smoke", vocab_size=1000, hidden_size=1024, num_layers=4, num_heads=16, q_lora_rank=256,
                      o_groups=4, o_lora_rank=256, compress_ratios=[0, 4, 128, 4], index_heads=8, index_topk=32,
                      n_routed_experts=8, moe_topk=2, moe_intermediate=1024, dense_format="bf16", max_position=8192)
    ecfg = EngineConfig(kv_cache_format="direct", max_running_requests=2, cuda_graph_bs=[1, 2],
                        chunked_prefill_size=256, enable_hierarchical_cache=True)
    eng = Engine.build(cfg, ecfg, device, max_context=1024, max_requests=2, kv_bytes=64 << 20)
    eng.runner.capture()
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(3, cfg.vocab_size, (300,), generator=g).tolist()
    out = eng.generate([prompt], SamplingParams(max_new_tokens=3))[0]
    out2 = eng.generate([prompt + out + [5, 6, 7]], SamplingParams(max_new_tokens=2))[0]  # restored from HiCache
    torch.cuda.synchronize(device)
    check_errors(device)
    eng.runner.release()
    assert len(out) == 3 and len(out2) == 2 and eng.metrics.snapshot().get("hicache_hit_tokens", 0) > 0

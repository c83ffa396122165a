"""HiCache on the GPU: the segment-copy kernel between device and pinned host memory, engine restore."""
import pytest
import torch

from packmla.ops._ext import check_errors, ext

pytestmark = pytest.mark.gpu


def test_segment_copy_round_trip(cuda):
    dev = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device=cuda)
    host = torch.zeros(1 << 20, dtype=torch.uint8, pin_memory=True)
    back = torch.zeros_like(dev)
    sizes = [16, 4096, 37376, 512, 65536, 1 << 18]
    segs, off = [], 0
    for n in sizes:
        segs.append([dev.data_ptr() + off, host.data_ptr() + off, n])
        off += n
    ext().segment_copy(torch.tensor(segs, dtype=torch.int64, device=cuda))
    torch.cuda.synchronize()
    assert torch.equal(host[:off], dev[:off].cpu())
    ext().segment_copy(torch.tensor([[host.data_ptr() + o, back.data_ptr() + o, n] for (_, _, n), o in
                                     zip(segs, [s[0] - dev.data_ptr() for s in segs])], dtype=torch.int64, device=cuda))
    torch.cuda.synchronize()
    assert torch.equal(back[:off], dev[:off])


@pytest.mark.parametrize("layout", ["page_first", "layer_first"])
def test_engine_restores_previous_turn(cuda, layout):
    from helpers import small_gpu_config

    from packmla.config import EngineConfig
    from packmla.engine.engine import Engine, SamplingParams

    cfg = small_gpu_config()
    ecfg = EngineConfig(kv_cache_format="direct", max_running_requests=2, cuda_graph_bs=[1, 2],
                        chunked_prefill_size=128, disable_cuda_graph=True, enable_hierarchical_cache=True,
                        hicache_mem_layout=layout)
    eng = Engine.build(cfg, ecfg, cuda, max_context=1024, max_requests=2, kv_bytes=64 << 20)
    g = torch.Generator().manual_seed(0)
    turn1 = torch.randint(3, cfg.vocab_size, (300,), generator=g).tolist()
    out1 = eng.generate([turn1], SamplingParams(max_new_tokens=4))[0]
    entry = next(iter(eng.hicache.entries.values()))
    slot = eng.pool.admit(400)
    eng.hicache.restore(entry, slot)
    torch.cuda.synchronize()
    for d, h in eng.hicache._segments(slot, len(entry.host_pages), len(entry.host_c128), entry):
        assert torch.equal(d.cpu(), h)
    eng.pool.release(slot)
    turn2 = turn1 + out1 + torch.randint(3, cfg.vocab_size, (20,), generator=g).tolist()
    out2 = eng.generate([turn2], SamplingParams(max_new_tokens=4))[0]
    check_errors(cuda)
    assert len(out2) == 4 and eng.metrics.snapshot()["hicache_hit_tokens"] == len(turn1) + len(out1) - 1

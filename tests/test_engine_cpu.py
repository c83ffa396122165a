"""CPU: model prefill/decode consistency, engine scheduling, capacity accounting."""
import pytest
import torch

from packmla.config import EngineConfig, ModelConfig
from packmla.engine.engine import Engine, SamplingParams
from packmla.kv.pool import KVPool, plan_capacity
from packmla.models.v4flash import V4FlashModel
from packmla.models.weights import init_weights


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def test_prefill_chunking_and_decode_agree():
    cfg = ModelConfig.tiny(num_layers=4)
    W = init_weights(cfg)
    for fmt in ("direct", "native", "fp4-native", "fp4-direct"):
        pool = KVPool(cfg, EngineConfig(kv_cache_format=fmt, device="cpu"), 16, 4, 1024, "cpu")
        m = V4FlashModel(cfg, W, pool)
        toks = torch.randint(0, cfg.vocab_size, (300,), generator=torch.Generator().manual_seed(0))
        s1 = pool.admit(300)
        full = m.prefill(toks, 0, s1)
        s2 = pool.admit(300)
        m.prefill(toks[:200], 0, s2)
        m.prefill(toks[200:299], 200, s2)
        step = m.decode(toks[299:300], torch.tensor([299]), torch.tensor([s2]))[0]
        assert _rel(step, full) < 2e-2


def test_engine_batch_invariance_and_metrics():
    cfg = ModelConfig.tiny(num_layers=3)
    ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=4, cuda_graph_bs=[1, 2, 4])
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 130, 5)]
    eng = Engine.build(cfg, ecfg, "cpu", max_context=512)
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=5))
    assert [len(o) for o in outs] == [5, 5, 5]
    alone = Engine.build(cfg, ecfg, "cpu", max_context=512).generate([prompts[1]], SamplingParams(max_new_tokens=5))
    assert alone[0] == outs[1]
    m = eng.metrics.snapshot()
    assert m["requests_finished"] == 3 and m["prefill_tokens"] == 205
    assert eng.pool.pages.free == eng.pool.num_pages  # all pages returned


def test_capacity_ratio_packed_vs_native():
    cfg = ModelConfig()
    budget = 30 << 30
    native = plan_capacity(cfg, EngineConfig(kv_cache_format="native"), budget)
    direct = plan_capacity(cfg, EngineConfig(kv_cache_format="direct"), budget)
    ratio = direct.max_total_tokens / native.max_total_tokens
    assert ratio >= 1.21, ratio


def test_engine_config_rejects_unsupported():
    import pytest

    with pytest.raises(ValueError):
        EngineConfig(kv_cache_format="direct", keep_count=192).validate()
    with pytest.raises(ValueError):
        EngineConfig(kv_cache_format="packed").validate()
    with pytest.raises(ValueError, match="HiCache"):
        EngineConfig(kv_cache_format="fp4-direct", enable_hierarchical_cache=True).validate()
    with pytest.raises(ValueError, match="adapter"):
        EngineConfig(kv_cache_format="fp4-direct", decode_impl="adapter").validate()
    with pytest.raises(ValueError):
        EngineConfig(kv_cache_format="native", enable_hierarchical_cache=True, keep_count=128).validate()


def test_pool_exhaustion_and_release():
    cfg = ModelConfig.tiny(num_layers=2)
    pool = KVPool(cfg, EngineConfig(device="cpu"), 4, 3, 2048, "cpu")
    s = pool.admit(700)  # 3 pages
    try:
        pool.admit(600)
        raise AssertionError("expected exhaustion")
    except MemoryError:
        pass
    pool.release(s)
    assert pool.pages.free == 4


def test_adapter_decode_matches_direct():
    """Adapter mode (Packed rows reconstructed as Native records before attention) gives the Direct
    mode's tokens: the reconstruction is lossless."""
    cfg = ModelConfig.tiny(num_layers=3)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (90, 150)]
    outs = {}
    for impl in ("direct", "adapter"):
        ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=2, cuda_graph_bs=[1, 2],
                            decode_impl=impl)
        outs[impl] = Engine.build(cfg, ecfg, "cpu", max_context=512).generate(prompts, SamplingParams(max_new_tokens=6))
    assert outs["adapter"] == outs["direct"]


def test_safetensors_checkpoint_round_trip(tmp_path):
    from packmla.models.weights import flatten, load_checkpoint, save_safetensors

    cfg = ModelConfig.tiny(num_layers=2)
    W = init_weights(cfg)
    names = save_safetensors(str(tmp_path / "ckpt"), W, cfg, shard_bytes=1 << 20)
    assert len(names) > 1  # sharded
    W2, cfg2 = load_checkpoint(str(tmp_path / "ckpt"))
    assert cfg2 == cfg and W2["meta"] == W["meta"]
    a, b = flatten(W), flatten(W2)
    assert set(a) == set(b) and all(torch.equal(a[k], b[k]) for k in a)
    # the receipt catches a changed shard before the weights are used
    shard = tmp_path / "ckpt" / names[0]
    data = bytearray(shard.read_bytes())
    data[-1] ^= 0x01
    shard.write_bytes(bytes(data))
    with pytest.raises(ValueError, match="changed"):
        load_checkpoint(str(tmp_path / "ckpt"))


def test_torch_checkpoint_round_trip_loads_weights_only(tmp_path):
    from packmla.models.weights import flatten, load_checkpoint, save_checkpoint

    cfg = ModelConfig.tiny(num_layers=2)
    W = init_weights(cfg)
    save_checkpoint(str(tmp_path / "w.pt"), W, cfg)
    W2, cfg2 = load_checkpoint(str(tmp_path / "w.pt"))
    a, b = flatten(W), flatten(W2)
    assert cfg2 == cfg and all(torch.equal(a[k], b[k]) for k in a)


def test_prefill_chunks_and_decode_steps_alternate():
    """A long prompt arriving while a request decodes must not stall that request's tokens until its
    whole prefill is done; the tokens themselves do not depend on the schedule."""
    cfg = ModelConfig.tiny(num_layers=2)
    g = torch.Generator().manual_seed(9)
    short = torch.randint(0, cfg.vocab_size, (20,), generator=g).tolist()
    long = torch.randint(0, cfg.vocab_size, (400,), generator=g).tolist()
    outs = {}
    for interleave in (True, False):
        ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=2, cuda_graph_bs=[1, 2],
                            prefill_decode_interleave=interleave)
        eng = Engine.build(cfg, ecfg, "cpu", max_context=1024)
        a = eng.add_request(short, SamplingParams(max_new_tokens=6))
        eng.step()  # prefill of the short prompt: it is now decoding
        b = eng.add_request(long, SamplingParams(max_new_tokens=2))
        kinds = []
        while eng.has_work():
            before = eng.metrics.snapshot().get("decode_steps", 0)
            eng.step()
            kinds.append("d" if eng.metrics.snapshot().get("decode_steps", 0) > before else "p")
        outs[interleave] = (eng.result(a).output_ids, eng.result(b).output_ids, "".join(kinds))
    assert outs[True][:2] == outs[False][:2]
    assert outs[True][2].startswith("dpdpdp")  # alternating while the long prompt is prefilled
    assert outs[False][2].startswith("ppppppp")  # prefill first: the short request waits


def test_per_layer_survivor_counts():
    """Per-layer Packed layouts: validation (adapter reads only, 64 .. 448 by 64, C4 layers only, no HiCache),
    capacity summing each layer's record size, and prefill chunking / decode agreement through
    reconstruction."""
    cfg = ModelConfig.tiny(num_layers=4)
    c4 = cfg.c4_layers
    counts = {layer: (128 if i % 2 == 0 else 448) for i, layer in enumerate(c4)}
    with pytest.raises(ValueError, match="256 only"):
        EngineConfig(layer_keep_counts=counts).validate()
    with pytest.raises(ValueError, match="steps of 64"):
        EngineConfig(decode_impl="adapter", layer_keep_counts={c4[0]: 100}).validate()
    with pytest.raises(ValueError, match="HiCache"):
        EngineConfig(decode_impl="adapter", layer_keep_counts=counts, enable_hierarchical_cache=True).validate()
    ecfg = EngineConfig(kv_cache_format="direct", decode_impl="adapter", layer_keep_counts=counts, device="cpu")
    ecfg.validate()
    non_c4 = next(i for i in range(cfg.num_layers) if i not in c4)
    with pytest.raises(ValueError, match="without C4"):
        KVPool(cfg, EngineConfig(decode_impl="adapter", layer_keep_counts={non_c4: 128}, device="cpu"), 4, 2, 512,
               "cpu")
    from packmla.kv.pool import bytes_per_full_token

    base = bytes_per_full_token(cfg, "direct", 0.1)
    mixed = bytes_per_full_token(cfg, "direct", 0.1, ecfg.keep_for)
    assert mixed - base == pytest.approx(sum(c - 256 for c in counts.values()) / 4)
    W = init_weights(cfg)
    pool = KVPool(cfg, ecfg, 16, 4, 1024, "cpu")
    assert {l: pool.c4_values[l].shape[1] for l in c4} == counts
    m = V4FlashModel(cfg, W, pool)
    toks = torch.randint(0, cfg.vocab_size, (300,), generator=torch.Generator().manual_seed(1))
    s1 = pool.admit(300)
    full = m.prefill(toks, 0, s1)
    s2 = pool.admit(300)
    m.prefill(toks[:200], 0, s2)
    m.prefill(toks[200:299], 200, s2)
    step = m.decode(toks[299:300], torch.tensor([299]), torch.tensor([s2]))[0]
    assert _rel(step, full) < 2e-2


def test_prompt_logprobs_match_direct_forward_and_chunking():
    """Prompt scoring (the completions `echo` + `logprobs`): the log-probability of prompt token i equals
    log-softmax of a direct prefill ending at token i - 1, whatever the chunk size; the top-k holds the
    most likely tokens; max_new_tokens = 0 generates nothing."""
    cfg = ModelConfig.tiny(num_layers=3)
    W = init_weights(cfg)
    prompt = torch.randint(3, cfg.vocab_size, (150,), generator=torch.Generator().manual_seed(5)).tolist()
    got = {}
    for chunk in (64, 256):
        ecfg = EngineConfig(device="cpu", chunked_prefill_size=chunk, max_running_requests=2, cuda_graph_bs=[1, 2],
                            prefix_cache=True)
        eng = Engine.build(cfg, ecfg, "cpu", max_context=512, weights=W)
        rid = eng.add_request(prompt, SamplingParams(max_new_tokens=0, prompt_logprobs=3))
        while eng.has_work():
            eng.step()
        r = eng.result(rid)
        assert r.output_ids == [] and len(r.prompt_lp) == len(prompt) and r.prompt_lp[0] is None
        got[chunk] = r
    a, b = got[64], got[256]
    assert max(abs(x - y) for x, y in zip(a.prompt_lp[1:], b.prompt_lp[1:])) < 2e-3
    for i in (1, 64, 65, 149):  # a chunk start, the first token of the second chunk, the last token
        pool = KVPool(cfg, EngineConfig(device="cpu"), 16, 2, 1024, "cpu")
        m = V4FlashModel(cfg, W, pool)
        logits = m.prefill(torch.tensor(prompt[:i]), 0, pool.admit(300))
        ref = (logits.log_softmax(-1)[prompt[i]]).item()
        assert abs(a.prompt_lp[i] - ref) < 2e-3, (i, a.prompt_lp[i], ref)
        top = a.prompt_top[i]
        assert len(top) == 3 and top[0][1] >= top[1][1] >= top[2][1] and a.prompt_lp[i] <= top[0][1] + 1e-5
        assert top[0][0] == int(logits.argmax())


def test_prompt_scoring_from_a_start_reuses_the_shared_prefix():
    """logprob_start_len: requests that share a long context and differ in their last tokens (the
    multiple-choice scoring of LongBench) reuse the context's prefix blocks and score only their tails,
    with the log-probabilities of a request scored in full."""
    cfg = ModelConfig.tiny(num_layers=3)
    W = init_weights(cfg)
    g = torch.Generator().manual_seed(8)
    ctx = torch.randint(3, cfg.vocab_size, (600,), generator=g).tolist()
    ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=2, cuda_graph_bs=[1, 2],
                        prefix_cache=True, prefix_block_tokens=256)
    eng = Engine.build(cfg, ecfg, "cpu", max_context=1024, weights=W)
    full = Engine.build(cfg, EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=2,
                                          cuda_graph_bs=[1, 2]), "cpu", max_context=1024, weights=W)
    for choice in (7, 8, 9):
        p = ctx + [choice, 5]
        rid = eng.add_request(p, SamplingParams(max_new_tokens=0, prompt_logprobs=0, prompt_logprobs_from=len(ctx)))
        ref = full.add_request(p, SamplingParams(max_new_tokens=0, prompt_logprobs=0))
        for e in (eng, full):
            while e.has_work():
                e.step()
        a, b = eng.result(rid), full.result(ref)
        assert all(v is None for v in a.prompt_lp[:len(ctx)]) and len(a.prompt_lp) == len(p)
        for i in (len(ctx), len(ctx) + 1):
            assert abs(a.prompt_lp[i] - b.prompt_lp[i]) < 2e-3
    assert eng.metrics.snapshot()["prefix_block_hit_tokens"] == 2 * 512  # the second and third requests

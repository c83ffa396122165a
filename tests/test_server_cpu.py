"""CPU: the OpenAI-compatible HTTP API over the engine driver (tiny random-init model)."""
import json
import threading

import pytest
import torch
from fastapi.testclient import TestClient

from packmla.config import EngineConfig, ModelConfig
from packmla.engine.engine import Engine, SamplingParams
from packmla.server.app import create_app
from packmla.server.driver import EngineDriver
from packmla.server.tokenizer import ByteTokenizer


@pytest.fixture(scope="module")
def served():
    cfg = ModelConfig.tiny(num_layers=2)
    ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=4, cuda_graph_bs=[1, 2, 4])
    eng = Engine.build(cfg, ecfg, "cpu", max_context=512)
    driver = EngineDriver(eng).start()
    tok = ByteTokenizer(cfg.vocab_size)
    app = create_app(driver, tok, "tiny")
    with TestClient(app) as client:
        yield client, eng, tok, cfg
    driver.stop()


def _reference_tokens(cfg, prompt, n):
    """Greedy tokens of the same model through a fresh engine (same seed => same weights)."""
    ecfg = EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=4, cuda_graph_bs=[1, 2, 4])
    eng = Engine.build(cfg, ecfg, "cpu", max_context=512)
    return eng.generate([prompt], SamplingParams(max_new_tokens=n, eos_token_id=2, ignore_eos=False))[0]


def test_health_models_info_metrics(served):
    client, eng, tok, cfg = served
    assert client.get("/health").text == "ok"
    assert client.get("/health_generate").status_code == 200
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    info = client.get("/server_info").json()
    assert info["kv_cache_format"] == "direct" and info["max_total_num_tokens"] > 0
    assert client.post("/flush_cache").status_code == 200
    assert "packmla_requests_finished" in client.get("/metrics").text


def test_completions_match_engine_generate(served):
    client, eng, tok, cfg = served
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "hello world", "max_tokens": 5})
    assert r.status_code == 200, r.text
    body = r.json()
    ids = body["choices"][0]["token_ids"]
    assert body["usage"] == {"prompt_tokens": 12, "completion_tokens": len(ids), "total_tokens": 12 + len(ids),
                             "prompt_tokens_details": {"cached_tokens": 0}}
    assert ids == _reference_tokens(cfg, tok.encode("hello world"), 5)
    assert body["choices"][0]["text"] == tok.decode(ids)
    # token-id prompt, two prompts in one call
    r2 = client.post("/v1/completions", json={"prompt": [tok.encode("hello world"), [1, 50, 60]], "max_tokens": 5})
    ch = r2.json()["choices"]
    assert ch[0]["token_ids"] == ids and len(ch) == 2


def test_streaming_completions_and_chat(served):
    client, eng, tok, cfg = served
    with client.stream("POST", "/v1/completions", json={"prompt": "stream me", "max_tokens": 4, "stream": True,
                                                       "ignore_eos": True}) as r:
        events = [l[6:] for l in r.iter_lines() if l.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    streamed = [c["choices"][0]["token_ids"][0] for c in chunks if c["choices"][0].get("token_ids")]
    assert len(streamed) == 4 and chunks[-1]["choices"][0]["finish_reason"] == "length"
    full = client.post("/v1/completions", json={"prompt": "stream me", "max_tokens": 4, "ignore_eos": True}).json()
    assert full["choices"][0]["token_ids"] == streamed

    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
    c = client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 3, "ignore_eos": True}).json()
    assert c["object"] == "chat.completion" and c["usage"]["completion_tokens"] == 3
    with client.stream("POST", "/v1/chat/completions", json={"messages": msgs, "max_tokens": 3, "stream": True,
                                                            "ignore_eos": True}) as r:
        ev = [json.loads(l[6:]) for l in r.iter_lines() if l.startswith("data: ") and l != "data: [DONE]"]
    text = "".join(e["choices"][0]["delta"].get("content", "") for e in ev)
    assert ev[0]["choices"][0]["delta"]["role"] == "assistant"
    assert text == c["choices"][0]["message"]["content"]


def test_generate_native_and_errors(served):
    client, eng, tok, cfg = served
    g = client.post("/generate", json={"input_ids": [1, 70, 80], "sampling_params": {"max_new_tokens": 2,
                                                                                    "ignore_eos": True}}).json()
    assert len(g["output_ids"]) == 2 and g["meta_info"]["prompt_tokens"] == 3
    assert client.post("/v1/completions", json={"prompt": "x", "max_tokens": 0}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": "x" * 600, "max_tokens": 4}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": [cfg.vocab_size + 5], "max_tokens": 1}).status_code == 400
    assert client.post("/v1/chat/completions", json={"messages": []}).status_code == 400


def test_concurrent_requests_batch_and_match(served):
    client, eng, tok, cfg = served
    prompts = ["alpha", "beta beta", "gamma gamma gamma"]
    out = {}

    def run(p):
        out[p] = client.post("/v1/completions", json={"prompt": p, "max_tokens": 6, "ignore_eos": True}
                             ).json()["choices"][0]["token_ids"]

    threads = [threading.Thread(target=run, args=(p,)) for p in prompts]
    before = eng.metrics.snapshot().get("decode_steps", 0)
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for p in prompts:
        ref = Engine.build(cfg, EngineConfig(device="cpu", chunked_prefill_size=64, max_running_requests=4,
                                             cuda_graph_bs=[1, 2, 4]), "cpu", max_context=512).generate(
            [tok.encode(p)], SamplingParams(max_new_tokens=6))[0]
        assert out[p] == ref
    assert eng.metrics.snapshot()["decode_steps"] - before < 3 * 5  # decode steps were shared


def test_stop_strings_stop_tokens_and_n(served):
    client, eng, tok, cfg = served
    base = client.post("/v1/completions", json={"prompt": "stop here", "max_tokens": 8, "ignore_eos": True}).json()
    ids = base["choices"][0]["token_ids"]
    # stop token: the output ends before its first occurrence, the request is cut short
    r = client.post("/v1/completions", json={"prompt": "stop here", "max_tokens": 8, "ignore_eos": True,
                                             "stop_token_ids": [ids[3]]}).json()["choices"][0]
    assert r["token_ids"] == ids[:ids.index(ids[3])] and r["finish_reason"] == "stop"
    # stop string: the text ends before it (same rule as the server: first completion of the string)
    stop = tok.decode([ids[4]])
    kept, expect = [], None
    for t in ids:
        full = tok.decode(kept + [t])
        if stop in full:
            expect = full[:full.find(stop)]
            break
        kept.append(t)
    r = client.post("/v1/completions", json={"prompt": "stop here", "max_tokens": 8, "ignore_eos": True,
                                             "stop": [stop]}).json()["choices"][0]
    assert r["text"] == expect and r["token_ids"] == kept and r["finish_reason"] == "stop"
    # streaming ends with finish_reason stop
    with client.stream("POST", "/v1/completions", json={"prompt": "stop here", "max_tokens": 8, "stream": True,
                                                       "ignore_eos": True, "stop_token_ids": [ids[3]]}) as s:
        ev = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ") and l != "data: [DONE]"]
    assert ev[-1]["choices"][0]["finish_reason"] == "stop"
    # n choices (greedy: identical), indexed in order
    c = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "max_tokens": 2,
                                                  "n": 3, "ignore_eos": True}).json()
    assert [ch["index"] for ch in c["choices"]] == [0, 1, 2] and c["usage"]["completion_tokens"] == 6
    assert len({ch["message"]["content"] for ch in c["choices"]}) == 1
    assert client.post("/v1/completions", json={"prompt": "x", "n": 17}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": "x", "stop": [3]}).status_code == 400


def test_profile_range_endpoints(served):
    import time

    client, eng, tok, cfg = served

    def wait_for(key, n):
        for _ in range(200):
            if eng.metrics.snapshot().get(key, 0) == n:
                return True
            time.sleep(0.02)
        return False

    assert client.post("/start_profile").status_code == 200
    assert wait_for("profile_ranges_opened", 1)
    client.post("/start_profile")  # already open: no second range
    assert client.post("/stop_profile").status_code == 200
    assert wait_for("profile_ranges_closed", 1)
    assert eng.metrics.snapshot()["profile_ranges_opened"] == 1
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "after profiling", "max_tokens": 2})
    assert r.status_code == 200


def test_unsupported_sampling_knobs_are_rejected(served):
    client, eng, tok, cfg = served
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "x", "max_tokens": 2, "top_p": 0.9})
    assert r.status_code == 400 and "top_p" in r.text
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "x", "max_tokens": 2, "top_p": 1.0,
                                             "top_k": -1, "frequency_penalty": 0})
    assert r.status_code == 200
    r = client.post("/generate", json={"text": "x", "sampling_params": {"max_new_tokens": 2, "top_k": 20}})
    assert r.status_code == 400


def test_event_loop_lag_probe_is_exported(served):
    import time

    client, eng, tok, cfg = served
    for _ in range(50):
        if "event_loop_lag_ms_max" in eng.metrics.snapshot():
            break
        time.sleep(0.05)
    text = client.get("/metrics").text
    assert "packmla_event_loop_lag_ms_last" in text and "packmla_event_loop_lag_ms_max" in text


def test_latency_histograms_on_metrics(served):
    client, eng, tok, cfg = served
    client.post("/v1/completions", json={"model": "tiny", "prompt": "histogram", "max_tokens": 3, "ignore_eos": True})
    text = client.get("/metrics").text
    for name in ("time_to_first_token_seconds", "e2e_request_latency_seconds", "time_per_output_token_seconds"):
        assert f'packmla_{name}_bucket{{le="+Inf"}}' in text and f"packmla_{name}_count" in text


def test_n_choices_share_one_prefill(served):
    client, eng, tok, cfg = served
    before = eng.metrics.snapshot().get("prefill_tokens", 0)
    body = {"model": "tiny", "prompt": "one prefill for three choices", "max_tokens": 4, "n": 3, "ignore_eos": True}
    c = client.post("/v1/completions", json=body).json()
    plen = c["usage"]["prompt_tokens"]
    assert len(c["choices"]) == 3 and len({ch["text"] for ch in c["choices"]}) == 1  # greedy copies agree
    assert eng.metrics.snapshot()["prefill_tokens"] - before == plen
    # the forks' copies of the leader's KV are not cache hits of the prompt: a fresh prompt has none
    cached = c["usage"]["prompt_tokens_details"]["cached_tokens"]
    assert cached <= plen and cached == 0
    assert eng.metrics.snapshot()["fork_copied_tokens"] >= 2 * plen


def test_streaming_with_n_choices(served):
    client, eng, tok, cfg = served
    for path, body in (("/v1/completions", {"prompt": "stream three", "max_tokens": 3, "ignore_eos": True}),
                       ("/v1/chat/completions", {"messages": [{"role": "user", "content": "stream three"}],
                                                 "max_tokens": 3, "ignore_eos": True})):
        r = client.post(path, json={"model": "tiny", "n": 3, "stream": True, **body})
        assert r.status_code == 200
        chunks = [json.loads(line[6:]) for line in r.text.splitlines()
                  if line.startswith("data: {")]
        assert r.text.rstrip().endswith("data: [DONE]")
        per = {i: [] for i in range(3)}
        finished = {}
        for c in chunks:
            ch = c["choices"][0]
            piece = ch.get("text") if "text" in ch else ch.get("delta", {}).get("content")
            if piece:
                per[ch["index"]].append(piece)
            if ch.get("finish_reason"):
                finished[ch["index"]] = ch["finish_reason"]
        assert finished == {0: "length", 1: "length", 2: "length"}
        assert all(len(v) == 3 for v in per.values()) and per[0] == per[1] == per[2]  # greedy copies
        usage = [c["usage"] for c in chunks if c.get("usage")]
        assert len(usage) == 1 and usage[0]["completion_tokens"] == 9


def test_api_key_guards_every_route_but_health():
    from packmla.server.app import create_app

    cfg = ModelConfig.tiny(num_layers=2)
    eng = Engine.build(cfg, EngineConfig(device="cpu", max_running_requests=2, cuda_graph_bs=[1, 2]), "cpu",
                       max_context=256)
    driver = EngineDriver(eng).start()
    try:
        with TestClient(create_app(driver, ByteTokenizer(cfg.vocab_size), "tiny", api_key="s3cret")) as client:
            assert client.get("/health").status_code == 200
            body = {"model": "tiny", "prompt": "x", "max_tokens": 1}
            assert client.post("/v1/completions", json=body).status_code == 401
            assert client.get("/v1/models", headers={"Authorization": "Bearer wrong"}).status_code == 401
            ok = client.post("/v1/completions", json=body, headers={"Authorization": "Bearer s3cret"})
            assert ok.status_code == 200
    finally:
        driver.stop()


def test_completions_echo_and_logprobs(served):
    """echo + logprobs + max_tokens 0 scores the prompt (the request lm-eval's log-likelihood tasks send);
    logprobs alone returns each generated token's log-probability."""
    client, eng, tok, cfg = served
    prompt = "the quick brown fox"
    ids = tok.encode(prompt)
    r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 0, "echo": True, "logprobs": 2})
    assert r.status_code == 200, r.text
    ch = r.json()["choices"][0]
    lp = ch["logprobs"]
    assert ch["token_ids"] == [] and ch["text"] == tok.decode(ids)
    assert len(lp["token_logprobs"]) == len(ids) and lp["token_logprobs"][0] is None
    assert all(v <= 0 for v in lp["token_logprobs"][1:])
    assert lp["top_logprobs"][0] is None and all(len(t) <= 2 for t in lp["top_logprobs"][1:])
    assert lp["text_offset"][0] == 0 and len(lp["tokens"]) == len(ids)
    r2 = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 3, "logprobs": 0})
    lp2 = r2.json()["choices"][0]["logprobs"]
    assert len(lp2["token_logprobs"]) == 3 and all(v <= 0 for v in lp2["token_logprobs"])
    assert client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 0}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": prompt, "logprobs": 99}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": prompt, "echo": True, "logprobs": 1,
                                                "stream": True}).status_code == 400


def test_longbench_evaluator_scores_choices_and_resumes(served, tmp_path):
    """The LongBench v2 evaluator over the HTTP API: each choice letter scored as a continuation (echo +
    logprobs + logprob_start_len), the best one predicted; results appended per item, a rerun skips the
    finished items; contexts beyond the limit are middle-truncated."""
    from packmla.bench import longbench

    client, eng, tok, cfg = served
    items = [{"_id": f"q{i}", "domain": "d", "sub_domain": "s", "difficulty": ("easy", "hard")[i % 2],
              "length": "short", "question": f"question {i}?", "choice_A": "a", "choice_B": "b", "choice_C": "c",
              "choice_D": "d", "answer": "ABCD"[i], "context": "lorem ipsum " * (10 + 5 * i)} for i in range(3)]
    data = tmp_path / "data.jsonl"
    data.write_text("\n".join(json.dumps(x) for x in items))

    def post(body):
        r = client.post("/v1/completions", json=body)
        assert r.status_code == 200, r.text
        return r.json()

    loaded = longbench.load_items(data)
    out = tmp_path / "run"
    s1 = longbench.evaluate(loaded, post, tok, out, max_prompt_tokens=300)
    rows = [json.loads(x) for x in (out / "items.jsonl").read_text().splitlines()]
    assert s1["overall"]["n"] == 3 and set(s1["difficulty"]) == {"easy", "hard"}
    assert all(set(r["scores"]) == set("ABCD") and r["pred"] == max(r["scores"], key=r["scores"].get) for r in rows)
    assert all(r["prompt_tokens"] <= 300 for r in rows)
    s2 = longbench.evaluate(loaded, post, tok, out, max_prompt_tokens=300)  # resumed: nothing new to score
    assert s2 == s1 and len((out / "items.jsonl").read_text().splitlines()) == 3
    g = longbench.evaluate(loaded[:1], post, tok, tmp_path / "gen", mode="generate")
    assert g["overall"]["n"] == 1
    assert longbench.parse_answer("The correct answer is (C).") == "C"


def test_chat_preparation_workers_and_frontend_diagnostics():
    """Chat conversion on a 2-worker pool gives the same tokens as inline conversion; diagnostics carry the
    preparation and first-output stamps in order; a conversion outlives a cancelled caller and keeps its
    admission until it ends."""
    import asyncio
    import time as _time

    from packmla.server.app import ChatPreparation

    cfg = ModelConfig.tiny(num_layers=2)
    eng = Engine.build(cfg, EngineConfig(device="cpu", max_running_requests=2, cuda_graph_bs=[1, 2]), "cpu",
                       max_context=256)
    driver = EngineDriver(eng).start()
    msgs = [{"role": "user", "content": "hello there"}]
    body = {"model": "tiny", "messages": msgs, "max_tokens": 3, "temperature": 0}
    outs = {}
    try:
        for workers, diag in ((0, False), (2, True)):
            app = create_app(driver, ByteTokenizer(cfg.vocab_size), "tiny", preparation_workers=workers,
                             frontend_diagnostics=diag)
            with TestClient(app) as client:
                r = client.post("/v1/chat/completions", json=body).json()
                outs[workers] = r["choices"][0]["message"]["content"]
                if diag:
                    d = r["diagnostics"]
                    order = ["preparation_queued_ms", "preparation_started_ms", "preparation_finished_ms",
                             "preparation_resumed_ms", "submitted_ms", "first_output_engine_ms",
                             "first_output_api_ms"]
                    assert [d[k] for k in order] == sorted(d[k] for k in order)
                    lines = [x for x in client.post("/v1/chat/completions", json={**body, "stream": True}).text
                             .splitlines() if x.startswith("data: {")]
                    assert "first_output_api_ms" in json.loads(lines[-1][6:])["diagnostics"]
                else:
                    assert "diagnostics" not in r
    finally:
        driver.stop()
    assert outs[0] == outs[2]

    release = threading.Event()

    def slow(m):
        release.wait(5)
        return [1, 2, 3]

    prep = ChatPreparation(slow, 1)

    async def scenario():
        first = asyncio.create_task(prep.prepare(["a"]))
        await asyncio.sleep(0.05)
        first.cancel()  # the caller goes away; the conversion keeps the single admission
        await asyncio.sleep(0.05)
        second = asyncio.create_task(prep.prepare(["b"]))
        await asyncio.sleep(0.1)
        assert not second.done()  # still waiting for the admission held by the running conversion
        release.set()
        ids, stamps = await asyncio.wait_for(second, 5)
        return ids, stamps

    t = _time.perf_counter()
    ids, stamps = asyncio.run(scenario())
    assert ids == [1, 2, 3] and stamps["queued"] >= t and stamps["resumed"] >= stamps["finished"]
    prep.close()
    with pytest.raises(ValueError):
        ChatPreparation(slow, 3)


def test_reasoning_parser_moves_the_think_block_to_reasoning_content():
    cfg = ModelConfig.tiny(num_layers=2)
    eng = Engine.build(cfg, EngineConfig(device="cpu", max_running_requests=2, cuda_graph_bs=[1, 2]), "cpu",
                       max_context=256)
    driver = EngineDriver(eng).start()
    body = {"model": "tiny", "messages": [{"role": "user", "content": "think"}], "max_tokens": 6, "temperature": 0}
    try:
        with TestClient(create_app(driver, ByteTokenizer(cfg.vocab_size), "tiny")) as plain_client:
            plain = plain_client.post("/v1/chat/completions", json=body).json()["choices"][0]["message"]
        assert "reasoning_content" not in plain
        app = create_app(driver, ByteTokenizer(cfg.vocab_size), "tiny", reasoning_parser="deepseek-v4")
        with TestClient(app) as client:
            think = {**body, "chat_template_kwargs": {"thinking": True}}
            msg = client.post("/v1/chat/completions", json=think).json()["choices"][0]["message"]
            # greedy output without an end tag: all of it is the open think block
            assert msg["reasoning_content"] == plain["content"] and msg["content"] == ""
            lines = [json.loads(x[6:]) for x in client.post("/v1/chat/completions", json={**think, "stream": True})
                     .text.splitlines() if x.startswith("data: {")]
            deltas = [c["choices"][0]["delta"] for c in lines]
            assert "".join(d.get("reasoning_content", "") for d in deltas) == plain["content"]
            assert not any(d.get("content") for d in deltas)
            off = client.post("/v1/chat/completions", json={**think, "separate_reasoning": False}).json()
            assert off["choices"][0]["message"]["content"] == plain["content"]
            no_think = client.post("/v1/chat/completions", json=body).json()["choices"][0]["message"]
            assert no_think["content"] == plain["content"] and no_think["reasoning_content"] == ""
    finally:
        driver.stop()

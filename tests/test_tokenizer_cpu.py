"""CPU: a local Hugging Face tokenizer (--tokenizer PATH) behind the server's tokenizer interface."""
import pytest


def _make_tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    words = ["<unk>", "<s>", "</s>", "hello", "world", "packed", "cache", "the", "is", "fast"]
    tk = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    fast = PreTrainedTokenizerFast(tokenizer_object=tk, bos_token="<s>", eos_token="</s>", unk_token="<unk>")
    fast.save_pretrained(str(path))


def test_hf_tokenizer_round_trip_and_server(tmp_path):
    from fastapi.testclient import TestClient

    from packmla.config import EngineConfig, ModelConfig
    from packmla.engine.engine import Engine
    from packmla.server.app import create_app
    from packmla.server.driver import EngineDriver
    from packmla.server.tokenizer import ByteTokenizer, HFTokenizer, load_tokenizer

    _make_tokenizer(tmp_path / "tok")
    tok = load_tokenizer(str(tmp_path / "tok"), 512)
    assert isinstance(tok, HFTokenizer) and isinstance(load_tokenizer(None, 512), ByteTokenizer)
    ids = tok.encode("the cache is fast")
    assert ids == [1, 7, 6, 8, 9] and tok.eos_token_id == 2
    assert tok.decode(ids[1:]) == "the cache is fast"
    assert tok.decode([3, 400]) == "hello"  # ids beyond the tokenizer (random-init samples) are dropped
    chat = tok.apply_chat_template([{"role": "user", "content": "hello world"}])
    assert 3 in chat and 4 in chat
    with pytest.raises(ValueError):
        HFTokenizer(str(tmp_path / "tok"), 5)  # more tokens than the model's vocabulary

    cfg = ModelConfig.tiny(num_layers=2)
    eng = Engine.build(cfg, EngineConfig(device="cpu", max_running_requests=2, cuda_graph_bs=[1, 2]), "cpu",
                       max_context=256)
    driver = EngineDriver(eng).start()
    try:
        with TestClient(create_app(driver, tok, "tiny")) as client:
            r = client.post("/v1/chat/completions", json={"model": "tiny", "max_tokens": 3,
                                                           "messages": [{"role": "user", "content": "hello"}]})
            assert r.status_code == 200 and r.json()["usage"]["completion_tokens"] <= 3
    finally:
        driver.stop()

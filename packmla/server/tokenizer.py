"""Byte-level tokenizer for random-init models (no tokenizer files exist offline).

Ids 0..2 are <pad>, <bos>, <eos>; id 3 + b encodes byte b.  Ids past the byte range (a random-init
model samples from the whole vocabulary) decode to the placeholder `<|id|>`, so every generated
token is visible in the text and `output_ids` stays exact.  The chat template is the plain
`<|role|>content` concatenation followed by `<|assistant|>`.
"""
from __future__ import annotations

PAD, BOS, EOS = 0, 1, 2
OFFSET = 3


class ByteTokenizer:
    def __init__(self, vocab_size: int):
        if vocab_size < OFFSET + 256:
            raise ValueError("vocab_size must hold the 256 byte tokens")
        self.vocab_size = vocab_size
        self.bos_token_id = BOS
        self.eos_token_id = EOS

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = [OFFSET + b for b in text.encode("utf-8")]
        return ([BOS] if add_bos else []) + ids

    def decode(self, ids: list[int]) -> str:
        out: list[str] = []
        buf = bytearray()
        for t in ids:
            if OFFSET <= t < OFFSET + 256:
                buf.append(t - OFFSET)
                continue
            if buf:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
            if t not in (PAD, BOS, EOS):
                out.append(f"<|{t}|>")
        if buf:
            out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)

    def apply_chat_template(self, messages: list[dict]) -> list[int]:
        text = "".join(f"<|{m.get('role', 'user')}|>{_content(m.get('content', ''))}" for m in messages)
        return self.encode(text + "<|assistant|>")


def _content(c) -> str:
    if isinstance(c, str):
        return c
    if isinstance(c, list):  # OpenAI content parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict))
    return str(c)


class HFTokenizer:
    """A local Hugging Face tokenizer (a checkpoint's tokenizer.json / tokenizer_config.json) behind the
    interface of `ByteTokenizer`; loaded with `local_files_only`, so nothing is downloaded.  The chat
    template is the tokenizer's own when it has one, else the plain concatenation above."""

    def __init__(self, path: str, vocab_size: int):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        if len(self.tok) > vocab_size:
            raise ValueError(f"tokenizer has {len(self.tok)} tokens, the model's vocabulary {vocab_size}")
        self.vocab_size = vocab_size
        self.bos_token_id = self.tok.bos_token_id if self.tok.bos_token_id is not None else 0
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = self.tok.encode(text, add_special_tokens=False)
        return ([self.bos_token_id] if add_bos and self.tok.bos_token_id is not None else []) + ids

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode([i for i in ids if i < len(self.tok)], skip_special_tokens=True)

    def apply_chat_template(self, messages: list[dict]) -> list[int]:
        msgs = [{"role": m.get("role", "user"), "content": _content(m.get("content", ""))} for m in messages]
        if getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True))
        return self.encode("".join(f"<|{m['role']}|>{m['content']}" for m in msgs) + "<|assistant|>")


def load_tokenizer(path: str | None, vocab_size: int):
    """`--tokenizer PATH` (a directory with Hugging Face tokenizer files), or the byte tokenizer."""
    return HFTokenizer(path, vocab_size) if path else ByteTokenizer(vocab_size)

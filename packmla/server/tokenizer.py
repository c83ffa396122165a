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

"""Reasoning parser: split a chat completion's text into `reasoning_content` and `content`.

Reference behaviour: the server is launched with `--reasoning-parser deepseek-v4` (or the GLM parser)
(scripts/local/run-server.sh:78-103), so chat responses carry the model's thinking apart from its answer,
as SGLang's reasoning parsers do.  The rule here, for the think-tag parsers:

* the think block is open from the start of the output when the template opens it in the prompt (the
  r1 parser, or a request with `chat_template_kwargs` `thinking` / `enable_thinking` true), or once the
  output begins with `<think>`; otherwise the whole output is the answer;
* inside an open block, text before the end tag `</think>` is reasoning and text after it is the answer;
  a block that never closes is all reasoning.

`ReasoningSplitter` applies the rule to streamed text: it holds back only the characters that could still
be the start of a tag, so deltas go out as soon as their side is known.
"""
from __future__ import annotations

PARSERS = {  # name -> (start tag, end tag, the chat template opens the block itself)
    "deepseek-v4": ("<think>", "</think>", False),
    "deepseek-v41": ("<think>", "</think>", False),
    "deepseek-r1": ("<think>", "</think>", True),
    "glm45": ("<think>", "</think>", False),
    "qwen3": ("<think>", "</think>", False),
}


def _tail_overlap(text: str, tag: str) -> int:
    """Length of the longest suffix of `text` that is a proper prefix of `tag`."""
    for n in range(min(len(tag) - 1, len(text)), 0, -1):
        if text.endswith(tag[:n]):
            return n
    return 0


class ReasoningSplitter:
    def __init__(self, parser: str, opened: bool | None = None):
        """`opened`: the prompt opened the think block (None: the parser's default)."""
        if parser not in PARSERS:
            raise ValueError(f"unknown reasoning parser {parser!r} (one of {', '.join(PARSERS)})")
        self.start, self.end, opens = PARSERS[parser]
        opens = opens if opened is None else opened
        self.state = "reasoning" if opens else "undecided"  # undecided -> reasoning | content
        self.buf = ""

    def feed(self, text: str) -> tuple[str, str]:
        """Append streamed text; returns the (reasoning, content) deltas that are settled."""
        self.buf += text
        reasoning = content = ""
        while True:
            if self.state == "undecided":
                stripped = self.buf.lstrip()
                if stripped.startswith(self.start):
                    self.buf = stripped[len(self.start):]
                    self.state = "reasoning"
                    continue
                if self.start.startswith(stripped):  # could still be the start tag
                    return reasoning, content
                self.state = "content"
                continue
            if self.state == "reasoning":
                i = self.buf.find(self.end)
                if i >= 0:
                    reasoning += self.buf[:i]
                    self.buf = self.buf[i + len(self.end):]
                    self.state = "content"
                    continue
                keep = _tail_overlap(self.buf, self.end)
                reasoning += self.buf[:len(self.buf) - keep]
                self.buf = self.buf[len(self.buf) - keep:]
                return reasoning, content
            content += self.buf
            self.buf = ""
            return reasoning, content

    def finish(self) -> tuple[str, str]:
        """End of output: whatever is held back goes to its side."""
        rest, self.buf = self.buf, ""
        if self.state == "reasoning":
            return rest, ""
        return "", rest


def opened_by_request(body: dict) -> bool | None:
    """Whether a chat request asked the template to open the think block (None: not said)."""
    kw = body.get("chat_template_kwargs") or {}
    for key in ("thinking", "enable_thinking"):
        if key in kw:
            return bool(kw[key])
    return None


def split(parser: str, text: str, opened: bool | None = None) -> tuple[str, str]:
    """(reasoning_content, content) of a whole output."""
    s = ReasoningSplitter(parser, opened)
    r1, c1 = s.feed(text)
    r2, c2 = s.finish()
    return r1 + r2, c1 + c2

"""CPU: the reasoning parser splits chat output into reasoning_content and content, whole or streamed."""
import random

import pytest

from packmla.server.reasoning import ReasoningSplitter, opened_by_request, split

CASES = [  # (parser, opened, text, reasoning, content)
    ("deepseek-v4", None, "<think>plan a</think>answer", "plan a", "answer"),
    ("deepseek-v4", None, "  <think>x</think>y", "x", "y"),
    ("deepseek-v4", None, "plain answer </think> stays", "", "plain answer </think> stays"),
    ("deepseek-v4", True, "thinking</think>done", "thinking", "done"),
    ("deepseek-r1", None, "r1 thought</think>r1 answer", "r1 thought", "r1 answer"),
    ("deepseek-v4", None, "<think>never closed", "never closed", ""),
    ("deepseek-v4", None, "<thi", "", "<thi"),
    ("deepseek-v4", None, "", "", ""),
    ("deepseek-r1", False, "no block</think>x", "", "no block</think>x"),
]


@pytest.mark.parametrize("parser,opened,text,reasoning,content", CASES)
def test_whole_and_streamed_outputs_split_alike(parser, opened, text, reasoning, content):
    assert split(parser, text, opened) == (reasoning, content)
    rng = random.Random(len(text))
    for _ in range(20):  # random chunkings of the same text
        s = ReasoningSplitter(parser, opened)
        r = c = ""
        i = 0
        while i < len(text):
            n = rng.randint(1, 4)
            dr, dc = s.feed(text[i:i + n])
            r, c, i = r + dr, c + dc, i + n
        dr, dc = s.finish()
        assert (r + dr, c + dc) == (reasoning, content)


def test_request_switch_and_unknown_parser():
    assert opened_by_request({"chat_template_kwargs": {"thinking": True}}) is True
    assert opened_by_request({"chat_template_kwargs": {"enable_thinking": False}}) is False
    assert opened_by_request({}) is None
    with pytest.raises(ValueError):
        ReasoningSplitter("nope")

"""LongBench v2 multiple-choice evaluation against a running packmla server.

    python -m packmla.bench.longbench data.json --url http://127.0.0.1:30000 --out results/lb2-direct \
        [--mode loglikelihood|generate] [--max-prompt-tokens 120000] [--tokenizer PATH] [--limit N]

Reference behaviour: scripts/local/bench-lb2.sh runs lm-eval's `longbench2` task through its
local-completions backend against the server's /v1/completions (a log-likelihood multiple-choice task,
resumable through lm-eval's request cache), comparing Native and Packed serving.  lm-eval is not part of
this environment, so packmla scores the same way itself:

  * `loglikelihood` (default): each item's prompt ends with "The correct answer is (", and every choice
    letter is scored as a continuation of it: one /v1/completions request per letter with `echo`,
    `logprobs: 0`, `max_tokens: 0` and SGLang's `logprob_start_len` at the continuation, so the four
    requests of an item share the long context through the server's prefix cache.  The prediction is the
    letter with the highest continuation log-probability.
  * `generate`: greedy completion of up to 32 tokens; the first "(X)" / letter A-D in it is the answer.

Data: the released LongBench v2 records (`data.json`, a JSON array, or JSONL) with fields `_id`, `domain`,
`sub_domain`, `difficulty` (easy / hard), `length` (short / medium / long), `question`, `choice_A` ..
`choice_D`, `answer` and `context`; read from a local file (no network).  Contexts longer than
`--max-prompt-tokens` keep their first and last halves, as LongBench truncates.  Per-item results are
appended to `<out>/items.jsonl` as they finish, and a rerun with the same `--out` skips the items already
there; `<out>/summary.json` gives the accuracy overall and by difficulty and length.
"""
from __future__ import annotations

import argparse
import json
import os
import re
from pathlib import Path

LETTERS = ("A", "B", "C", "D")
TEMPLATE = ("Please read the following text and answer the question below.\n\n<text>\n{context}\n</text>\n\n"
            "What is the correct answer to this question: {question}\nChoices:\n(A) {A}\n(B) {B}\n(C) {C}\n(D) {D}\n\n"
            "Format your response as follows: \"The correct answer is (insert answer here)\".")
ANSWER_PREFIX = "\nThe correct answer is ("


def load_items(path: Path) -> list[dict]:
    text = Path(path).read_text()
    items = json.loads(text) if text.lstrip().startswith("[") else [json.loads(x) for x in text.splitlines() if x.strip()]
    need = {"_id", "question", "choice_A", "choice_B", "choice_C", "choice_D", "answer", "context"}
    for it in items:
        missing = need - set(it)
        if missing:
            raise ValueError(f"record {it.get('_id', '?')} lacks {sorted(missing)}")
        if it["answer"] not in LETTERS:
            raise ValueError(f"record {it['_id']}: answer must be one of A-D")
    return items


def prompt_ids(item: dict, tokenizer, max_tokens: int | None) -> list[int]:
    """The item's prompt as token ids, its context middle-truncated to fit `max_tokens` in all."""
    def render(context: str) -> list[int]:
        return tokenizer.encode(TEMPLATE.format(context=context, question=item["question"],
                                                A=item["choice_A"], B=item["choice_B"], C=item["choice_C"],
                                                D=item["choice_D"]) + ANSWER_PREFIX)
    ids = render(item["context"])
    if max_tokens is None or len(ids) <= max_tokens:
        return ids
    ctx = tokenizer.encode(item["context"])
    keep = max(0, len(ctx) - (len(ids) - max_tokens))
    return render(tokenizer.decode(ctx[:keep // 2]) + tokenizer.decode(ctx[len(ctx) - (keep - keep // 2):]))


def parse_answer(text: str) -> str | None:
    m = re.search(r"\(([ABCD])\)", text) or re.search(r"\b([ABCD])\b", text)
    return m.group(1) if m else None


def score_item(post, item: dict, ids: list[int], tokenizer, mode: str) -> dict:
    """`post(body) -> response JSON` of /v1/completions."""
    if mode == "generate":
        out = post({"prompt": ids, "max_tokens": 32, "temperature": 0.0})
        text = out["choices"][0]["text"]
        pred = parse_answer(text)
        return {"pred": pred, "response": text}
    scores = {}
    for letter in LETTERS:
        cont = tokenizer.encode(letter)
        out = post({"prompt": ids + cont, "max_tokens": 0, "echo": True, "logprobs": 0,
                    "logprob_start_len": len(ids), "temperature": 0.0})
        lps = out["choices"][0]["logprobs"]["token_logprobs"][len(ids):]
        scores[letter] = float(sum(lps))
    pred = max(LETTERS, key=lambda x: scores[x])
    return {"pred": pred, "scores": scores}


def summarize(rows: list[dict]) -> dict:
    def acc(sel):
        sel = list(sel)
        return {"n": len(sel), "accuracy": round(sum(r["correct"] for r in sel) / len(sel), 4) if sel else None}

    out = {"overall": acc(rows)}
    for key in ("difficulty", "length"):
        out[key] = {v: acc(r for r in rows if r.get(key) == v) for v in sorted({r.get(key) for r in rows} - {None})}
    return out


def evaluate(items: list[dict], post, tokenizer, out_dir: Path, mode: str = "loglikelihood",
             max_prompt_tokens: int | None = None) -> dict:
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    log = out_dir / "items.jsonl"
    done = {}
    if log.exists():
        for line in log.read_text().splitlines():
            if line.strip():
                r = json.loads(line)
                done[r["_id"]] = r
    with open(log, "a") as f:
        for item in items:
            if item["_id"] in done:
                continue
            ids = prompt_ids(item, tokenizer, max_prompt_tokens)
            res = score_item(post, item, ids, tokenizer, mode)
            row = {"_id": item["_id"], "domain": item.get("domain"), "difficulty": item.get("difficulty"),
                   "length": item.get("length"), "answer": item["answer"], "prompt_tokens": len(ids),
                   "mode": mode, **res, "correct": res["pred"] == item["answer"]}
            f.write(json.dumps(row) + "\n")
            f.flush()
            done[item["_id"]] = row
    rows = [done[i["_id"]] for i in items if i["_id"] in done]
    summary = {"mode": mode, **summarize(rows)}
    tmp = out_dir / "summary.json.tmp"
    tmp.write_text(json.dumps(summary, indent=1) + "\n")
    os.replace(tmp, out_dir / "summary.json")
    return summary


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("data", type=Path)
    ap.add_argument("--url", default="http://127.0.0.1:30000")
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--mode", default="loglikelihood", choices=["loglikelihood", "generate"])
    ap.add_argument("--max-prompt-tokens", type=int, default=None)
    ap.add_argument("--tokenizer", default=None, help="the server's tokenizer (default: its byte tokenizer)")
    ap.add_argument("--vocab", type=int, default=129280)
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--model", default="default")
    args = ap.parse_args(argv)

    import requests

    from ..server.tokenizer import load_tokenizer
    from .serving import auth_headers

    tokenizer = load_tokenizer(args.tokenizer, args.vocab)
    items = load_items(args.data)[:args.limit]

    def post(body: dict) -> dict:
        r = requests.post(args.url + "/v1/completions", json={"model": args.model, **body},
                          headers=auth_headers(), timeout=3600)
        r.raise_for_status()
        return r.json()

    summary = evaluate(items, post, tokenizer, args.out, args.mode, args.max_prompt_tokens)
    print(json.dumps(summary))
    return summary


if __name__ == "__main__":
    main()

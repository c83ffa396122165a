"""Convert recorded agent traffic (LongSWE-style raw JSONL) into packmla's replay and request files.

    python -m packmla.bench.convert --input raw.jsonl --output-dir prepared/

Reference behaviour: scripts/local/convert_lswb.py (`prepare`, `prepare_replay`).  A raw record is
one JSON object per line:

    {"id": "req-1", "token_name": "user-7", "created": 1760000000.5,
     "messages": [{"role": "user", "content": "..."}, ...], "tools": [...],
     "usage": {"prompt_tokens": 31000, "completion_tokens": 412}}

`token_name` names the session (user); a record without one is a session of its own.  Every record
is validated (unique non-empty id, non-empty messages with string roles, a usage object, integer
token counts, a finite `created`, tools as a list) and any failure names the source line.  The output
directory must not exist; it is assembled under a temporary name and renamed into place:

    sessions.jsonl   replay input (`python -m packmla.bench.replay`): sessions ordered by their first
                     request's (created, id), turns by (created, id); max_tokens = the recorded
                     completion tokens (256 where none were recorded), ignore_eos false
    requests.jsonl   the same requests one per line in source order, for request-level clients
    manifest.json    source path and sha256, counts, and per request its source line, sha256 of the
                     source line, the output cap and whether the 256 default was used
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import shutil
import tempfile
from collections import defaultdict
from pathlib import Path

DEFAULT_OUTPUT_CAP = 256


def _int(value, where: str, name: str) -> int:
    if not isinstance(value, int) or isinstance(value, bool) or value < 0:
        raise ValueError(f"{where}: {name} must be an integer >= 0, got {value!r}")
    return value


def parse_record(raw: bytes, where: str) -> dict:
    """One raw line -> a validated request dict (raises ValueError naming `where`)."""
    try:
        doc = json.loads(raw)
    except (ValueError, UnicodeError) as exc:
        raise ValueError(f"{where}: invalid JSON: {exc}") from exc
    if not isinstance(doc, dict):
        raise ValueError(f"{where}: expected a JSON object")
    rid = doc.get("id")
    if not isinstance(rid, str) or not rid:
        raise ValueError(f"{where}: id must be a non-empty string")
    msgs = doc.get("messages")
    if not isinstance(msgs, list) or not msgs or any(
            not isinstance(m, dict) or not isinstance(m.get("role"), str) for m in msgs):
        raise ValueError(f"{where} ({rid}): messages must be a non-empty list of objects with a string role")
    usage = doc.get("usage")
    if not isinstance(usage, dict):
        raise ValueError(f"{where} ({rid}): usage must be an object")
    completion = usage.get("completion_tokens")
    prompt = usage.get("prompt_tokens")
    if completion is not None:
        _int(completion, f"{where} ({rid})", "completion_tokens")
    if prompt is not None:
        _int(prompt, f"{where} ({rid})", "prompt_tokens")
    session = doc.get("token_name")
    if session is not None and (not isinstance(session, str) or not session):
        raise ValueError(f"{where} ({rid}): token_name must be a non-empty string")
    created = doc.get("created")
    if not isinstance(created, (int, float)) or isinstance(created, bool) or not math.isfinite(created):
        raise ValueError(f"{where} ({rid}): created must be a finite number")
    tools = doc.get("tools")
    if tools is not None and not isinstance(tools, list):
        raise ValueError(f"{where} ({rid}): tools must be a list")
    return {"id": rid, "session": session or rid, "created": float(created), "messages": msgs,
            "tools": tools or None, "completion_tokens": completion, "prompt_tokens": prompt}


def convert(input_path: str, output_dir: str) -> dict:
    src = Path(input_path).resolve(strict=True)
    out = Path(output_dir).resolve()
    if out.exists():
        raise ValueError(f"{out} exists: choose a fresh output directory")
    out.parent.mkdir(parents=True, exist_ok=True)
    scratch = Path(tempfile.mkdtemp(prefix=".convert-", dir=out.parent))
    digest = hashlib.sha256()
    seen: set[str] = set()
    reqs: list[dict] = []
    entries: list[dict] = []
    try:
        with open(src, "rb") as f:
            for n, raw in enumerate(f, 1):
                digest.update(raw)
                if not raw.strip():
                    continue
                rec = parse_record(raw, f"{src}:{n}")
                if rec["id"] in seen:
                    raise ValueError(f"{src}:{n}: duplicate request id {rec['id']!r}")
                seen.add(rec["id"])
                cap = rec["completion_tokens"] or DEFAULT_OUTPUT_CAP
                rec["max_tokens"] = cap
                reqs.append(rec)
                entries.append({"request_id": rec["id"], "session": rec["session"], "source_line": n,
                                "source_sha256": hashlib.sha256(raw).hexdigest(), "max_tokens": cap,
                                "used_default_output_cap": not rec["completion_tokens"],
                                "recorded_prompt_tokens": rec["prompt_tokens"]})
        if not reqs:
            raise ValueError(f"{src}: no records")
        groups: dict[str, list[dict]] = defaultdict(list)
        for r in reqs:
            groups[r["session"]].append(r)
        for g in groups.values():
            g.sort(key=lambda r: (r["created"], r["id"]))
        order = sorted(groups, key=lambda s: (groups[s][0]["created"], groups[s][0]["id"], s))

        def line(r: dict, turn: int | None) -> str:
            body = {"session": r["session"], "request_id": r["id"], "messages": r["messages"],
                    "max_tokens": r["max_tokens"], "temperature": 0, "ignore_eos": False}
            if turn is not None:
                body["turn"] = turn
            if r["prompt_tokens"] is not None:
                body["prompt_tokens"] = r["prompt_tokens"]
            if r["tools"]:
                body["tools"] = r["tools"]
            return json.dumps(body, ensure_ascii=False, allow_nan=False, separators=(",", ":")) + "\n"

        with open(scratch / "sessions.jsonl", "w", encoding="utf-8") as f:
            for s in order:
                for t, r in enumerate(groups[s]):
                    f.write(line(r, t))
        with open(scratch / "requests.jsonl", "w", encoding="utf-8") as f:
            for r in reqs:
                f.write(line(r, None))
        manifest = {"source_path": str(src), "source_sha256": digest.hexdigest(), "requests": len(reqs),
                    "sessions": len(groups), "default_output_cap": DEFAULT_OUTPUT_CAP, "records": entries}
        (scratch / "manifest.json").write_text(json.dumps(manifest, indent=2, allow_nan=False) + "\n")
        os.rename(scratch, out)
    finally:
        if scratch.exists():
            shutil.rmtree(scratch)
    return {"output_dir": str(out), "requests": len(reqs), "sessions": len(groups)}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--input", required=True)
    ap.add_argument("--output-dir", required=True)
    a = ap.parse_args(argv)
    out = convert(a.input, a.output_dir)
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()

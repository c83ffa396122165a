"""OpenAI-compatible HTTP API over an `EngineDriver` (FastAPI).

Endpoints (reference server: SGLang OpenAI entrypoints + native routes used by the reference's
scripts, `scripts/local/env.sh:53-71` `health`, `scripts/local/bench-serving.sh` `--flush-cache`,
server-info records in every benchmark directory):

    GET  /health, /health_generate     liveness; the second runs a one-token generation
    GET  /v1/models
    POST /v1/completions               prompt: str | [str] | [int] | [[int]]; stream via SSE
    POST /v1/chat/completions          messages; stream via SSE (chat.completion.chunk deltas)
    POST /generate                     SGLang native: text | input_ids + sampling_params
    GET  /server_info (/get_server_info)
    POST /flush_cache
    GET  /metrics                      Prometheus text
"""
from __future__ import annotations

import asyncio
import json
import time
import uuid

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.engine import SamplingParams
from .driver import EngineDriver
from .tokenizer import ByteTokenizer


def _params(body: dict, tok: ByteTokenizer, default_max: int = 16) -> SamplingParams:
    max_tokens = body.get("max_completion_tokens", body.get("max_tokens", body.get("max_new_tokens", default_max)))
    if max_tokens is None or int(max_tokens) < 1:
        raise HTTPException(400, "max_tokens must be >= 1")
    temp = float(body.get("temperature", 0.0) or 0.0)
    if temp < 0:
        raise HTTPException(400, "temperature must be >= 0")
    return SamplingParams(max_new_tokens=int(max_tokens), temperature=temp,
                          ignore_eos=bool(body.get("ignore_eos", False)), eos_token_id=tok.eos_token_id)


def _prompts(prompt, tok: ByteTokenizer) -> list[list[int]]:
    if isinstance(prompt, str):
        return [tok.encode(prompt)]
    if isinstance(prompt, list) and prompt and all(isinstance(t, int) for t in prompt):
        return [list(prompt)]
    if isinstance(prompt, list) and prompt and all(isinstance(p, str) for p in prompt):
        return [tok.encode(p) for p in prompt]
    if isinstance(prompt, list) and prompt and all(isinstance(p, list) for p in prompt):
        return [list(p) for p in prompt]
    raise HTTPException(400, "prompt must be a string, a list of strings, or token ids")


def _check_ids(ids: list[int], vocab: int) -> None:
    if not ids or any((not isinstance(t, int)) or t < 0 or t >= vocab for t in ids):
        raise HTTPException(400, f"token ids must be non-empty and in [0, {vocab})")


def _sse(obj) -> bytes:
    return f"data: {json.dumps(obj)}\n\n".encode()


def create_app(driver: EngineDriver, tokenizer: ByteTokenizer, model_name: str, server_args: dict | None = None
               ) -> FastAPI:
    app = FastAPI(title="packmla")
    eng = driver.engine
    vocab = eng.cfg.vocab_size

    async def _submit(ids: list[int], params: SamplingParams):
        _check_ids(ids, vocab)
        try:
            return driver.submit(ids, params, asyncio.get_running_loop())
        except ValueError as exc:
            raise HTTPException(400, str(exc)) from exc
        except RuntimeError as exc:
            raise HTTPException(503, str(exc)) from exc

    async def _collect(st) -> list[int]:
        while True:
            item = await st.queue.get()
            if item is None:
                break
        if st.finish_reason == "error":
            raise HTTPException(500, f"engine failed: {driver.error!r}")
        return st.tokens

    def _usage(prompt_tokens: int, completion_tokens: int) -> dict:
        return {"prompt_tokens": prompt_tokens, "completion_tokens": completion_tokens,
                "total_tokens": prompt_tokens + completion_tokens}

    @app.get("/health")
    async def health():
        if driver.error is not None:
            return PlainTextResponse(f"engine failed: {driver.error!r}", status_code=503)
        if driver.stalled():
            return PlainTextResponse("engine step exceeded the watchdog timeout", status_code=503)
        return PlainTextResponse("ok")

    @app.get("/health_generate")
    async def health_generate():
        st = await _submit([tokenizer.bos_token_id], SamplingParams(max_new_tokens=1, ignore_eos=True))
        await _collect(st)
        return PlainTextResponse("ok")

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "packmla",
                                            "max_model_len": eng.pool.max_context}]}

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        params = _params(body, tokenizer)
        prompts = _prompts(body.get("prompt"), tokenizer)
        rid = f"cmpl-{uuid.uuid4().hex}"
        created = int(time.time())
        if body.get("stream"):
            if len(prompts) != 1:
                raise HTTPException(400, "streaming supports one prompt")
            st = await _submit(prompts[0], params)

            async def gen():
                n = 0
                while True:
                    item = await st.queue.get()
                    if item is None:
                        break
                    n += 1
                    yield _sse({"id": rid, "object": "text_completion", "created": created, "model": model_name,
                                "choices": [{"index": 0, "text": tokenizer.decode([item]), "token_ids": [item],
                                             "logprobs": None, "finish_reason": None}]})
                yield _sse({"id": rid, "object": "text_completion", "created": created, "model": model_name,
                            "choices": [{"index": 0, "text": "", "logprobs": None,
                                         "finish_reason": st.finish_reason}],
                            "usage": _usage(st.prompt_len, n)})
                yield b"data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        streams = [await _submit(p, params) for p in prompts]
        choices = []
        ntok = 0
        for i, st in enumerate(streams):
            toks = await _collect(st)
            ntok += len(toks)
            choices.append({"index": i, "text": tokenizer.decode(toks), "token_ids": toks, "logprobs": None,
                            "finish_reason": st.finish_reason})
        return {"id": rid, "object": "text_completion", "created": created, "model": model_name,
                "choices": choices, "usage": _usage(sum(len(p) for p in prompts), ntok)}

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise HTTPException(400, "messages must be a non-empty list")
        params = _params(body, tokenizer)
        ids = tokenizer.apply_chat_template(msgs)
        rid = f"chatcmpl-{uuid.uuid4().hex}"
        created = int(time.time())
        st = await _submit(ids, params)
        if body.get("stream"):
            async def gen():
                yield _sse({"id": rid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                            "choices": [{"index": 0, "delta": {"role": "assistant"}, "finish_reason": None}]})
                n = 0
                while True:
                    item = await st.queue.get()
                    if item is None:
                        break
                    n += 1
                    yield _sse({"id": rid, "object": "chat.completion.chunk", "created": created,
                                "model": model_name,
                                "choices": [{"index": 0, "delta": {"content": tokenizer.decode([item])},
                                             "finish_reason": None}]})
                yield _sse({"id": rid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                            "choices": [{"index": 0, "delta": {}, "finish_reason": st.finish_reason}],
                            "usage": _usage(len(ids), n)})
                yield b"data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        toks = await _collect(st)
        return {"id": rid, "object": "chat.completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "message": {"role": "assistant", "content": tokenizer.decode(toks)},
                             "finish_reason": st.finish_reason}],
                "usage": _usage(len(ids), len(toks))}

    @app.post("/generate")
    async def generate(req: Request):
        body = await req.json()
        sp = dict(body.get("sampling_params") or {})
        params = _params(sp, tokenizer)
        if "input_ids" in body:
            ids = list(body["input_ids"])
        elif isinstance(body.get("text"), str):
            ids = tokenizer.encode(body["text"])
        else:
            raise HTTPException(400, "give text or input_ids")
        st = await _submit(ids, params)
        toks = await _collect(st)
        now = time.perf_counter()
        return {"text": tokenizer.decode(toks), "output_ids": toks,
                "meta_info": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                              "finish_reason": {"type": st.finish_reason},
                              "e2e_latency": now - st.t_submit,
                              "ttft": (st.t_first - st.t_submit) if st.t_first else None}}

    @app.get("/server_info")
    @app.get("/get_server_info")
    async def server_info():
        info = dict(eng.server_info())
        info.update({"model_path": model_name, "model_config": json.loads(eng.cfg.to_json()),
                     "capacity": eng.capacity.as_dict(), **(server_args or {})})
        return JSONResponse(info)

    @app.post("/flush_cache")
    async def flush_cache():
        driver.flush_cache()
        return PlainTextResponse("Cache flushed.")

    @app.get("/metrics")
    async def metrics():
        m = eng.metrics
        m.set("num_running_reqs", len(eng.running))
        m.set("num_queue_reqs", len(eng.waiting))
        m.set("kv_pages_free", eng.pool.pages.free)
        return PlainTextResponse(m.prometheus())

    return app

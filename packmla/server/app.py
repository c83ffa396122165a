"""OpenAI-compatible HTTP API over an `EngineDriver` (FastAPI).

Endpoints (reference server: SGLang OpenAI entrypoints + native routes used by the reference's
scripts, `scripts/local/env.sh:53-71` `health`, `scripts/local/bench-serving.sh` `--flush-cache`,
server-info records in every benchmark directory):

    GET  /health, /health_generate     liveness; the second runs a one-token generation
    GET  /v1/models
    POST /v1/completions               prompt: str | [str] | [int] | [[int]]; n; stop / stop_token_ids; SSE
    POST /v1/chat/completions          messages; n; stop / stop_token_ids; SSE (chat.completion.chunk deltas)

A stop string or stop token ends a choice early (the engine request is aborted) and is not returned.
While streaming, text already sent before a multi-token stop string completes is not withdrawn.
    POST /generate                     SGLang native: text | input_ids + sampling_params
    GET  /server_info (/get_server_info)
    POST /flush_cache
    POST /start_profile, /stop_profile  CUDA profiler capture range (Nsight --capture-range=cudaProfilerApi)
    GET  /metrics                      Prometheus text
"""
from __future__ import annotations

import asyncio
import contextlib
import json
import time
import uuid

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.engine import SamplingParams
from .driver import EngineDriver
from .tokenizer import ByteTokenizer


def _logprobs_args(body: dict) -> tuple[bool, int | None]:
    """(echo, logprobs) of a completions request: `logprobs` k in [0, 20] returns each token's
    log-probability and, for prompt positions (with echo), the top k there."""
    echo = bool(body.get("echo", False))
    k = body.get("logprobs")
    if k is not None and (isinstance(k, bool) or not isinstance(k, int) or not 0 <= k <= 20):
        raise HTTPException(400, "logprobs must be an integer in [0, 20]")
    if (echo or k is not None) and body.get("stream"):
        raise HTTPException(400, "echo and logprobs are returned by non-streaming requests only")
    return echo, k


def _start_len(body: dict) -> int:
    """SGLang's `logprob_start_len`: prompt tokens before it are not scored (and may come from a cache)."""
    v = body.get("logprob_start_len", 0)
    if v is None:
        return 0
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise HTTPException(400, "logprob_start_len must be an integer >= 0")
    return v


def _params(body: dict, tok: ByteTokenizer, default_max: int = 16, scoring: tuple | None = None) -> SamplingParams:
    max_tokens = body.get("max_completion_tokens", body.get("max_tokens", body.get("max_new_tokens", default_max)))
    echo, k = scoring if scoring is not None else (False, None)
    if max_tokens is None or int(max_tokens) < (0 if echo else 1):
        raise HTTPException(400, "max_tokens must be >= 1 (>= 0 with echo)")
    temp = float(body.get("temperature", 0.0) or 0.0)
    if temp < 0:
        raise HTTPException(400, "temperature must be >= 0")
    sp = body.get("sampling_params") if isinstance(body.get("sampling_params"), dict) else body
    # the sampler is greedy or temperature-scaled over the full vocabulary; other knobs are rejected rather
    # than silently ignored (their neutral values pass)
    for name, neutral in (("top_p", 1.0), ("top_k", -1), ("min_p", 0.0), ("frequency_penalty", 0.0),
                          ("presence_penalty", 0.0), ("repetition_penalty", 1.0)):
        v = sp.get(name)
        if v is not None and not (v == neutral or (name == "top_k" and v == 0)):
            raise HTTPException(400, f"{name}={v} is not supported (greedy or temperature sampling only)")
    return SamplingParams(max_new_tokens=int(max_tokens), temperature=temp,
                          ignore_eos=bool(body.get("ignore_eos", False)), eos_token_id=tok.eos_token_id,
                          prompt_logprobs=(k or 0) if echo and k is not None else None, logprobs=k is not None,
                          prompt_logprobs_from=_start_len(body))


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


class _StopRule:
    """OpenAI `stop` strings and `stop_token_ids` of one choice: the token that completes a stop string,
    or a stop token, ends the choice and is not returned; the text ends before the stop string."""

    def __init__(self, body: dict, tok: ByteTokenizer):
        stop = body.get("stop")
        strings = [stop] if isinstance(stop, str) else list(stop or [])
        if not all(isinstance(x, str) for x in strings):
            raise HTTPException(400, "stop must be a string or a list of strings")
        self.strings = [x for x in strings if x]
        try:
            self.ids = {int(t) for t in (body.get("stop_token_ids") or [])}
        except (TypeError, ValueError) as exc:
            raise HTTPException(400, "stop_token_ids must be token ids") from exc
        self.tok = tok
        self.tokens: list[int] = []
        self.text: str | None = None  # final text when a stop string ended the choice

    @property
    def active(self) -> bool:
        return bool(self.strings or self.ids)

    def accept(self, token: int) -> bool:
        if token in self.ids:
            return False
        if self.strings:
            full = self.tok.decode(self.tokens + [token])
            hits = [full.find(x) for x in self.strings if x in full]
            if hits:
                self.text = full[:min(hits)]
                return False
        self.tokens.append(token)
        return True


def _sse(obj) -> bytes:
    return f"data: {json.dumps(obj)}\n\n".encode()


class ChatPreparation:
    """Chat-template conversion of a request's messages, inline (no worker, the default) or on a pool of
    1, 2 or 4 worker threads with admission bounded by the pool size.

    Reference behaviour: SGLang's opt-in `SGLANG_DSV4_ASYNC_PREPARATION` text-chat worker with
    `DSV4_PREPARATION_WORKERS=1|2|4` (third_party/README.md:310-323): conversion leaves the API event loop;
    a cancelled request keeps its admission until its conversion completes; shutdown drains owned work;
    off creates no worker.  `prepare` returns the token ids and, in perf_counter seconds, the stamps
    queued / started / finished / resumed (the last when the API coroutine runs again)."""

    def __init__(self, convert, workers: int = 0):
        if workers not in (0, 1, 2, 4):
            raise ValueError("chat preparation workers must be 0 (inline), 1, 2 or 4")
        self.convert = convert
        self.workers = workers
        self._pool = None
        self._admission: asyncio.Semaphore | None = None
        if workers:
            from concurrent.futures import ThreadPoolExecutor

            self._pool = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="chat-prep")

    def _run(self, msgs, stamps: dict):
        stamps["started"] = time.perf_counter()
        try:
            return self.convert(msgs)
        finally:
            stamps["finished"] = time.perf_counter()

    async def prepare(self, msgs) -> tuple[list[int], dict]:
        stamps = {"queued": time.perf_counter()}
        if self._pool is None:
            return self._run(msgs, stamps), stamps
        if self._admission is None:
            self._admission = asyncio.Semaphore(self.workers)
        await self._admission.acquire()
        fut = asyncio.get_running_loop().run_in_executor(self._pool, self._run, msgs, stamps)
        # the admission is released when the conversion ends, not when a cancelled caller stops waiting
        fut.add_done_callback(lambda _f: self._admission.release())
        ids = await asyncio.shield(fut)
        stamps["resumed"] = time.perf_counter()
        return ids, stamps

    def close(self) -> None:
        if self._pool is not None:
            self._pool.shutdown(wait=True)  # drain conversions still running


def _diagnostics(t0: float, prep: dict, st, api_first: float | None) -> dict:
    """First-output diagnostics in ms after the API handler started (fields that never happened stay absent)."""
    out = {f"preparation_{k}_ms": round((v - t0) * 1e3, 3) for k, v in prep.items()}
    if st is not None and st.t_submit:
        out["submitted_ms"] = round((st.t_submit - t0) * 1e3, 3)
    if st is not None and st.t_first is not None:
        out["first_output_engine_ms"] = round((st.t_first - t0) * 1e3, 3)
    if api_first is not None:
        out["first_output_api_ms"] = round((api_first - t0) * 1e3, 3)
    return out


def create_app(driver: EngineDriver, tokenizer: ByteTokenizer, model_name: str, server_args: dict | None = None,
               api_key: str | None = None, preparation_workers: int = 0,
               frontend_diagnostics: bool = False, reasoning_parser: str | None = None) -> FastAPI:
    """`api_key`: when set, every route but /health answers 401 unless the request carries
    `Authorization: Bearer <api_key>` (SGLang's --api-key).  `preparation_workers`: chat-template
    conversion on 1, 2 or 4 worker threads (0: inline).  `frontend_diagnostics`: chat responses carry a
    `diagnostics` object with preparation and first-output stamps.  `reasoning_parser`: chat messages
    carry the output's think block as `reasoning_content` (a request may send `separate_reasoning` false)."""
    eng = driver.engine
    vocab = eng.cfg.vocab_size
    prep = ChatPreparation(tokenizer.apply_chat_template, preparation_workers)
    if reasoning_parser is not None:
        from .reasoning import PARSERS

        if reasoning_parser not in PARSERS:
            raise ValueError(f"unknown reasoning parser {reasoning_parser!r}")

    @contextlib.asynccontextmanager
    async def lifespan(_app):
        # event-loop lag probe (reference: its frontend event-loop probe): a 100 ms sleep that wakes late
        # means request handlers or token delivery are blocking the loop
        async def probe():
            loop = asyncio.get_running_loop()
            worst = 0.0
            while True:
                t = loop.time()
                await asyncio.sleep(0.1)
                lag = max(0.0, (loop.time() - t - 0.1) * 1000)
                worst = max(worst, lag)
                eng.metrics.set("event_loop_lag_ms_last", round(lag, 3))
                eng.metrics.set("event_loop_lag_ms_max", round(worst, 3))

        task = asyncio.create_task(probe())
        try:
            yield
        finally:
            task.cancel()
            prep.close()

    app = FastAPI(title="packmla", lifespan=lifespan)

    if api_key:
        import hmac

        @app.middleware("http")
        async def require_key(request: Request, call_next):
            if request.url.path != "/health":
                given = request.headers.get("authorization", "")
                if not hmac.compare_digest(given.encode(), f"Bearer {api_key}".encode()):
                    return JSONResponse({"error": "invalid or missing API key"}, status_code=401)
            return await call_next(request)

    async def _submit(ids: list[int], params: SamplingParams):
        _check_ids(ids, vocab)
        try:
            return driver.submit(ids, params, asyncio.get_running_loop())
        except ValueError as exc:
            raise HTTPException(400, str(exc)) from exc
        except RuntimeError as exc:
            raise HTTPException(503, str(exc)) from exc

    async def _submit_group(ids: list[int], params: SamplingParams, n: int):
        """n choices of one prompt: prefilled once, the other choices copy its KV."""
        _check_ids(ids, vocab)
        try:
            return driver.submit_group(ids, params, n, asyncio.get_running_loop())
        except ValueError as exc:
            raise HTTPException(400, str(exc)) from exc
        except RuntimeError as exc:
            raise HTTPException(503, str(exc)) from exc

    async def _merge(streams, body: dict):
        """Events of several streams as they arrive: ("tok", index, token) and, once per stream after its
        last token, ("end", index, None).  Leaving early cancels the readers, whose requests are aborted."""
        q: asyncio.Queue = asyncio.Queue()

        async def pump(i, st):
            try:
                async for item in _tokens(st, _StopRule(body, tokenizer)):
                    q.put_nowait(("tok", i, item))
            finally:
                q.put_nowait(("end", i, None))

        tasks = [asyncio.create_task(pump(i, st)) for i, st in enumerate(streams)]
        ended = 0
        try:
            while ended < len(streams):
                ev = await q.get()
                ended += ev[0] == "end"
                yield ev
        finally:
            for t in tasks:
                t.cancel()

    async def _tokens(st, rule: _StopRule | None):
        """Tokens of one request as they arrive; a stop rule that fires aborts the request early, and so
        does a consumer that goes away first (a client that disconnected, a cancelled handler)."""
        stopped = ended = False
        try:
            while True:
                item = await st.queue.get()
                if item is None:
                    ended = True
                    break
                if stopped:
                    continue  # produced before the abort reached the engine
                if rule is not None and rule.active and not rule.accept(item):
                    stopped = True
                    driver.abort(st.ext_id)
                    continue
                yield item
        finally:
            if not ended and not stopped:
                driver.abort(st.ext_id)
        if stopped:
            st.finish_reason = "stop"

    async def _collect(st, rule: _StopRule | None = None) -> list[int]:
        toks = [t async for t in _tokens(st, rule)]
        if st.finish_reason == "error":
            raise HTTPException(500, f"engine failed: {driver.error!r}")
        return toks

    def _text(toks: list[int], rule: _StopRule | None) -> str:
        return rule.text if rule is not None and rule.text is not None else tokenizer.decode(toks)

    def _n(body: dict) -> int:
        n = body.get("n", 1)
        if not isinstance(n, int) or not 1 <= n <= 16:
            raise HTTPException(400, "n must be an integer in [1, 16]")
        return n

    def _cached(streams: list, n_choices: int) -> int:
        """Prompt tokens served from a cache, counted once per prompt.

        The streams of one prompt are its leader followed by its n - 1 forks; the forks copy the leader's
        prefilled KV, which is not a cache hit of the prompt, so only the leaders' counts are summed."""
        return sum(st.cached_tokens for st in streams[::max(1, n_choices)])

    def _usage(prompt_tokens: int, completion_tokens: int, cached_tokens: int = 0) -> dict:
        return {"prompt_tokens": prompt_tokens, "completion_tokens": completion_tokens,
                "total_tokens": prompt_tokens + completion_tokens,
                "prompt_tokens_details": {"cached_tokens": cached_tokens}}

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

    def _logprobs_obj(prompt: list[int], toks: list[int], st, echo: bool, k: int) -> dict:
        """The OpenAI completions `logprobs` object of one choice (prompt tokens first with echo)."""
        lp = st.logprobs or {}
        ids = (list(prompt) if echo else []) + list(toks)
        values = (list(lp.get("prompt_lp", [])) if echo else []) + list(lp.get("output_lp", []))[:len(toks)]
        top = None
        if k:
            top = [None if t is None else {tokenizer.decode([i]): v for i, v in t}
                   for t in (lp.get("prompt_top", []) if echo else [])]
            top += [{tokenizer.decode([t]): v} for t, v in zip(toks, lp.get("output_lp", []))]
        strs = [tokenizer.decode([t]) for t in ids]
        offsets, pos = [], 0
        for x in strs:
            offsets.append(pos)
            pos += len(x)
        return {"tokens": strs, "token_logprobs": values, "top_logprobs": top, "text_offset": offsets}

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        echo, k = _logprobs_args(body)
        params = _params(body, tokenizer, scoring=(echo, k))
        prompts = _prompts(body.get("prompt"), tokenizer)
        n_choices = _n(body)
        _StopRule(body, tokenizer)  # validate before submitting anything
        rid = f"cmpl-{uuid.uuid4().hex}"
        created = int(time.time())
        if body.get("stream"):
            if len(prompts) != 1:
                raise HTTPException(400, "streaming supports one prompt")
            streams = await _submit_group(prompts[0], params, n_choices)

            async def gen():
                n, ended = 0, 0
                async for kind, i, item in _merge(streams, body):
                    if kind == "tok":
                        n += 1
                        yield _sse({"id": rid, "object": "text_completion", "created": created, "model": model_name,
                                    "choices": [{"index": i, "text": tokenizer.decode([item]), "token_ids": [item],
                                                 "logprobs": None, "finish_reason": None}]})
                        continue
                    ended += 1
                    last = {"usage": _usage(len(prompts[0]), n, _cached(streams, n_choices))} \
                        if ended == len(streams) else {}
                    yield _sse({"id": rid, "object": "text_completion", "created": created, "model": model_name,
                                "choices": [{"index": i, "text": "", "logprobs": None,
                                             "finish_reason": streams[i].finish_reason}], **last})
                yield b"data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        streams = [st for p in prompts for st in await _submit_group(p, params, n_choices)]
        owners = [p for p in prompts for _ in range(n_choices)]
        choices = []
        ntok = 0
        for i, st in enumerate(streams):
            rule = _StopRule(body, tokenizer)
            toks = await _collect(st, rule)
            ntok += len(toks)
            text = _text(toks, rule)
            if echo:
                text = tokenizer.decode(owners[i]) + text
            choices.append({"index": i, "text": text, "token_ids": toks,
                            "logprobs": _logprobs_obj(owners[i], toks, st, echo, k) if k is not None else None,
                            "finish_reason": st.finish_reason})
        return {"id": rid, "object": "text_completion", "created": created, "model": model_name,
                "choices": choices,
                "usage": _usage(sum(len(p) for p in prompts), ntok, _cached(streams, n_choices))}

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        t0 = time.perf_counter()
        body = await req.json()
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise HTTPException(400, "messages must be a non-empty list")
        params = _params(body, tokenizer)
        n_choices = _n(body)
        _StopRule(body, tokenizer)
        ids, stamps = await prep.prepare(msgs)
        eng.metrics.observe("chat_preparation_seconds", stamps["finished"] - stamps["started"])
        api_first = [None]
        parser = reasoning_parser if body.get("separate_reasoning", True) else None
        rid = f"chatcmpl-{uuid.uuid4().hex}"
        created = int(time.time())
        if body.get("stream"):
            streams = await _submit_group(ids, params, n_choices)

            async def gen():
                from .reasoning import ReasoningSplitter, opened_by_request

                splitters = [ReasoningSplitter(parser, opened_by_request(body)) if parser else None
                             for _ in streams]

                def delta_chunk(i, reasoning: str, content: str) -> bytes | None:
                    delta = {k: v for k, v in (("reasoning_content", reasoning), ("content", content)) if v}
                    if not delta:
                        return None
                    return _sse({"id": rid, "object": "chat.completion.chunk", "created": created,
                                 "model": model_name, "choices": [{"index": i, "delta": delta, "finish_reason": None}]})

                for i in range(len(streams)):
                    yield _sse({"id": rid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                                "choices": [{"index": i, "delta": {"role": "assistant"}, "finish_reason": None}]})
                n, ended = 0, 0
                async for kind, i, item in _merge(streams, body):
                    if kind == "tok":
                        n += 1
                        if api_first[0] is None:
                            api_first[0] = time.perf_counter()
                        text = tokenizer.decode([item])
                        chunk = (delta_chunk(i, *splitters[i].feed(text)) if splitters[i] is not None
                                 else delta_chunk(i, "", text))
                        if chunk is not None:
                            yield chunk
                        continue
                    if splitters[i] is not None:
                        chunk = delta_chunk(i, *splitters[i].finish())
                        if chunk is not None:
                            yield chunk
                    ended += 1
                    last = {"usage": _usage(len(ids), n, _cached(streams, n_choices))} \
                        if ended == len(streams) else {}
                    if last and frontend_diagnostics:
                        last["diagnostics"] = _diagnostics(t0, stamps, streams[0], api_first[0])
                    yield _sse({"id": rid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                                "choices": [{"index": i, "delta": {}, "finish_reason": streams[i].finish_reason}],
                                **last})
                yield b"data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        streams = await _submit_group(ids, params, n_choices)
        choices, ntok = [], 0
        for i, st in enumerate(streams):
            rule = _StopRule(body, tokenizer)
            toks = []
            async for t in _tokens(st, rule):
                if api_first[0] is None:
                    api_first[0] = time.perf_counter()
                toks.append(t)
            if st.finish_reason == "error":
                raise HTTPException(500, f"engine failed: {driver.error!r}")
            ntok += len(toks)
            text = _text(toks, rule)
            message = {"role": "assistant", "content": text}
            if parser:
                from .reasoning import opened_by_request, split

                message["reasoning_content"], message["content"] = split(parser, text, opened_by_request(body))
            choices.append({"index": i, "message": message, "finish_reason": st.finish_reason})
        out = {"id": rid, "object": "chat.completion", "created": created, "model": model_name,
               "choices": choices, "usage": _usage(len(ids), ntok, _cached(streams, n_choices))}
        if frontend_diagnostics:
            out["diagnostics"] = _diagnostics(t0, stamps, streams[0], api_first[0])
        return out

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
        rule = _StopRule(sp, tokenizer)
        toks = await _collect(st, rule)
        now = time.perf_counter()
        return {"text": _text(toks, rule), "output_ids": toks,
                "meta_info": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                              "cached_tokens": st.cached_tokens,
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

    @app.post("/start_profile")
    async def start_profile():
        driver.profile(True)
        return PlainTextResponse("Start profiling.")

    @app.post("/stop_profile")
    async def stop_profile():
        driver.profile(False)
        return PlainTextResponse("Stop profiling.")

    @app.get("/metrics")
    async def metrics():
        m = eng.metrics
        m.set("num_running_reqs", len(eng.running))
        m.set("num_queue_reqs", len(eng.waiting))
        m.set("kv_pages_free", eng.pool.pages.free)
        return PlainTextResponse(m.prometheus())

    return app

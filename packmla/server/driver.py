"""Engine driver: the one thread that owns an `Engine`, fed by HTTP handlers through queues.

Reference behaviour (SGLang scheduler process behind the tokenizer manager): requests enter a
queue, the scheduler loop admits them and steps the model, and tokens stream back per request.
Here the loop runs on a thread of the server process; handlers await per-request asyncio queues
that the loop fills with `loop.call_soon_threadsafe`.

Tensor parallelism: rank 0 serves HTTP and, once per loop iteration, broadcasts the operations it
applies (add / abort / flush / stop) to the other ranks over a CPU (gloo) group; every rank applies
the same operations in the same order and then takes the same `Engine.step()`, so the schedules
and the KV pools stay identical in lockstep (reference: Gloo CPU broadcast of the batch each step).
With DP attention each request is served by one rank, so after every step the ranks' produced tokens
(with their finish state) are gathered to rank 0 over the same CPU group.
"""
from __future__ import annotations

import asyncio
import itertools
import queue
import threading
import time
from dataclasses import dataclass, field

from ..engine.engine import Engine, SamplingParams


@dataclass
class Stream:
    """Handle of one submitted request: tokens arrive on `queue`; `None` marks the end."""

    ext_id: int
    prompt_len: int
    loop: asyncio.AbstractEventLoop | None
    queue: asyncio.Queue | None
    tokens: list[int] = field(default_factory=list)
    finish_reason: str | None = None
    done: threading.Event = field(default_factory=threading.Event)
    t_submit: float = 0.0
    t_first: float | None = None
    params: SamplingParams | None = None
    prompt: list[int] | None = None  # kept only when the request log records prompt ids
    cached_tokens: int = 0  # prompt tokens served from a KV cache tier (known when the request ends)
    logprobs: dict | None = None  # prompt / output log-probabilities, when requested (set when it ends)


class EngineDriver:
    IDLE_WAIT_S = 0.02

    def __init__(self, engine: Engine, rank: int = 0, world: int = 1, cpu_group=None, watchdog_s: float = 1800.0,
                 error_check_every: int = 16, fault_hook=None, request_logger=None):
        """`watchdog_s`: a step running longer marks the server unhealthy (reference: --watchdog-timeout);
        `error_check_every`: steps between reads of the kernels' device error word (CUDA engines);
        `fault_hook(step)`: host-side fault injection for tests, called before every step;
        `request_logger`: a `RequestLogger` given every finished request."""
        self.engine = engine
        self.request_logger = request_logger
        self.watchdog_s = watchdog_s
        self.error_check_every = error_check_every
        self.fault_hook = fault_hook
        self.steps = 0
        self._step_started: float | None = None
        self.rank = rank
        self._last_work = False
        self.world = world
        self.cpu_group = cpu_group
        self._inbox: queue.Queue = queue.Queue()
        self._streams: dict[int, Stream] = {}
        self._rid_to_ext: dict[int, int] = {}
        self._ext_ids = itertools.count()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.error: BaseException | None = None

    # ------------------------------------------------------------------ public (any thread)
    def start(self) -> "EngineDriver":
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="packmla-engine", daemon=True)
            self._thread.start()
        return self

    def stop(self, timeout: float = 30.0) -> None:
        self._inbox.put(("stop",))
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout)

    def submit(self, prompt: list[int], params: SamplingParams, loop: asyncio.AbstractEventLoop | None = None
               ) -> Stream:
        if self.error is not None:
            raise RuntimeError(f"engine loop failed: {self.error!r}")
        if not prompt:
            raise ValueError("empty prompt")
        need = len(prompt) + params.max_new_tokens
        if need > self.engine.pool.max_context:
            raise ValueError(f"prompt + max_tokens = {need} exceeds the context limit {self.engine.pool.max_context}")
        ext = next(self._ext_ids)
        keep_prompt = self.request_logger is not None and self.request_logger.log_level >= 3
        st = Stream(ext, len(prompt), loop, asyncio.Queue() if loop is not None else None, t_submit=time.perf_counter(),
                    params=params, prompt=list(prompt) if keep_prompt else None)
        self._streams[ext] = st
        self._inbox.put(("add", ext, list(prompt), params))
        return st

    def submit_group(self, prompt: list[int], params: SamplingParams, n: int,
                     loop: asyncio.AbstractEventLoop | None = None) -> list[Stream]:
        """`n` streams of one prompt, prefilled once (the other requests copy its KV)."""
        if n <= 1:
            return [self.submit(prompt, params, loop)]
        if self.error is not None:
            raise RuntimeError(f"engine loop failed: {self.error!r}")
        if not prompt:
            raise ValueError("empty prompt")
        need = len(prompt) + params.max_new_tokens
        if need > self.engine.pool.max_context:
            raise ValueError(f"prompt + max_tokens = {need} exceeds the context limit {self.engine.pool.max_context}")
        streams = []
        for _ in range(n):
            ext = next(self._ext_ids)
            st = Stream(ext, len(prompt), loop, asyncio.Queue() if loop is not None else None,
                        t_submit=time.perf_counter(), params=params)
            self._streams[ext] = st
            streams.append(st)
        self._inbox.put(("add_group", [st.ext_id for st in streams], list(prompt), params))
        return streams

    def stalled(self) -> bool:
        t = self._step_started
        return t is not None and time.perf_counter() - t > self.watchdog_s

    def healthy(self) -> bool:
        return self.error is None and not self.stalled()

    def abort(self, ext: int) -> None:
        self._inbox.put(("abort", ext))

    def flush_cache(self) -> None:
        self._inbox.put(("flush",))

    def profile(self, on: bool) -> None:
        """Open or close the profiler capture range on every rank, between engine steps."""
        self._inbox.put(("profile", bool(on)))

    def generate(self, prompt: list[int], params: SamplingParams, timeout: float = 600.0) -> Stream:
        """Blocking convenience: submit and wait for the end of the request."""
        st = self.submit(prompt, params)
        if not st.done.wait(timeout):
            raise TimeoutError("request did not finish")
        return st

    # ------------------------------------------------------------------ engine thread
    def _collect_ops(self) -> list[tuple]:
        ops = []
        # the work state of the loop's last has_work(): under DP attention that call is a collective, which
        # only the loop may make (every rank makes it once per iteration)
        block = not self._last_work
        try:
            ops.append(self._inbox.get(timeout=self.IDLE_WAIT_S) if block else self._inbox.get_nowait())
            while True:
                ops.append(self._inbox.get_nowait())
        except queue.Empty:
            pass
        return ops

    def _sync_ops(self, ops: list[tuple]) -> list[tuple]:
        if self.world == 1:
            return ops
        import torch.distributed as dist

        box = [ops if self.rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=self.cpu_group)
        return box[0]

    def _apply(self, ops: list[tuple]) -> bool:
        eng = self.engine
        for op in ops:
            kind = op[0]
            if kind == "stop":
                return False
            if kind == "add":
                _, ext, prompt, params = op
                rid = eng.add_request(prompt, params)
                self._rid_to_ext[rid] = ext
            elif kind == "add_group":
                _, exts, prompt, params = op
                for rid, ext in zip(eng.add_group(prompt, params, len(exts)), exts):
                    self._rid_to_ext[rid] = ext
            elif kind == "abort":
                ext = op[1]
                for rid, e in list(self._rid_to_ext.items()):
                    if e == ext and eng.abort(rid):
                        eng.done.pop(rid, None)
                        self._finish(rid, "abort")
            elif kind == "flush":
                flush = getattr(eng, "flush_cache", None)
                if flush is not None:
                    flush()
            elif kind == "profile":
                eng.profile(op[1])
        return True

    def _finish(self, rid: int, reason: str) -> None:
        ext = self._rid_to_ext.pop(rid, None)
        st = self._streams.pop(ext, None) if ext is not None else None
        if st is None:
            return
        st.finish_reason = reason
        st.done.set()
        self._deliver_to(st, None)
        self._log(st)

    def _log(self, st: Stream) -> None:
        if self.request_logger is not None:
            try:
                self.request_logger.finished(st, st.prompt)
            except OSError:  # a full or vanished export directory must not stop serving
                self.engine.metrics.inc("request_log_errors")

    def _deliver_to(self, st: Stream, item) -> None:
        if st.queue is not None and st.loop is not None:
            st.loop.call_soon_threadsafe(st.queue.put_nowait, item)

    def _run(self, reraise: bool = False) -> None:
        eng = self.engine
        try:
            while True:
                ops = self._collect_ops() if self.rank == 0 else []
                ops = self._sync_ops(ops)
                if not self._apply(ops):
                    break
                self._last_work = eng.has_work()
                if not self._last_work:
                    continue
                self._step_started = time.perf_counter()
                if self.fault_hook is not None:
                    self.fault_hook(self.steps)
                produced = eng.step()
                self.steps += 1
                if eng.device.type == "cuda" and self.steps % self.error_check_every == 0:
                    from ..ops._ext import check_errors

                    check_errors(eng.device)  # a kernel's bounded wait or bounds check failed: stop serving
                self._step_started = None
                events = []
                for rid, tok in produced:
                    req = eng.done.pop(rid, None)  # the driver keeps no history of finished requests
                    fin = req is not None and req.finished
                    p = req.params if fin else None
                    hit_eos = bool(fin and not p.ignore_eos and p.eos_token_id is not None and req.output_ids
                                   and req.output_ids[-1] == p.eos_token_id)
                    scored = fin and (p.prompt_logprobs is not None or p.logprobs)
                    extra = {"prompt_lp": req.prompt_lp, "prompt_top": req.prompt_top,
                             "output_lp": req.output_lp} if scored else None
                    events.append((rid, tok, fin, hit_eos, req.cached_tokens if fin else 0, extra))
                if getattr(eng, "dp", False):  # every rank's tokens reach the HTTP streams on rank 0
                    import torch.distributed as dist

                    gathered = [None] * self.world
                    dist.all_gather_object(gathered, events, group=self.cpu_group)
                    events = [e for evs in gathered for e in evs]
                for rid, tok, fin, hit_eos, cached, extra in events:
                    ext = self._rid_to_ext.get(rid)
                    st = self._streams.get(ext) if ext is not None else None
                    if st is not None:
                        if st.t_first is None:
                            st.t_first = time.perf_counter()
                            eng.metrics.inc("ttft_seconds_sum", st.t_first - st.t_submit)
                            eng.metrics.observe("time_to_first_token_seconds", st.t_first - st.t_submit)
                        if tok is not None:  # None: a prompt-scoring request that generates nothing
                            st.tokens.append(tok)
                            self._deliver_to(st, tok)
                        if extra is not None:
                            st.logprobs = extra
                    if fin:
                        if st is not None:
                            st.cached_tokens = cached
                            now = time.perf_counter()
                            eng.metrics.inc("e2e_seconds_sum", now - st.t_submit)
                            eng.metrics.observe("e2e_request_latency_seconds", now - st.t_submit)
                            if st.t_first is not None and len(st.tokens) > 1:
                                eng.metrics.observe("time_per_output_token_seconds",
                                                    (now - st.t_first) / (len(st.tokens) - 1))
                        self._finish(rid, "stop" if hit_eos else "length")
        except BaseException as exc:  # surface to handlers instead of dying silently
            self.error = exc
            self._step_started = None
            eng.metrics.inc("engine_failures")
            for ext, st in list(self._streams.items()):
                st.finish_reason = "error"
                st.done.set()
                self._deliver_to(st, None)
                self._log(st)
            self._streams.clear()
            if reraise:
                raise

    def run_worker(self) -> None:
        """Ranks > 0: follow rank 0's operations until it sends `stop` (errors propagate to the caller)."""
        self._run(reraise=True)

"""Serving engine: requests, FCFS scheduler with chunked prefill, CUDA-graph decode runner.

Public API (what the HTTP server and bench.py call):

    eng = Engine.build(model_cfg, engine_cfg, device)            # random-init weights, KV pool
    rid = eng.add_request(prompt_ids, SamplingParams(max_new_tokens=256))
    while eng.has_work(): eng.step()                             # one prefill chunk or one decode step
    eng.result(rid).output_ids

Reference behaviour: SGLang scheduler + `decode_cuda_graph_runner.py` (third_party/README.md:294-298):
chunked prefill (8192), full decode CUDA graphs for padded batch sizes, FCFS admission bounded by
the KV pool.  Multi-rank: every rank runs the same deterministic schedule in lockstep; logits are
identical on all ranks after the all-reduces, so sampling needs no broadcast.  With DP attention
(`EngineConfig.dp_attention`) request rid belongs to rank rid % world, which alone schedules and serves it;
the ranks agree on each step's kind (prefill chunks or one decode step) and token counts through one
small exchange per step, because every MoE block exchanges tokens between them.
"""
from __future__ import annotations

import contextlib
import itertools
import os
import time
from collections import OrderedDict, deque
from dataclasses import dataclass, field

import torch

from ..config import EngineConfig, ModelConfig
from ..kv.pool import KVPool, plan_capacity
from ..models.v4flash import V4FlashModel
from ..models.weights import init_weights
from ..utils.metrics import Metrics


# NVTX ranges around scheduler steps and graph replays (PACKMLA_NVTX=1; reference: SGLang's
# SGLANG_ENABLE_NVTX_SCHEDULER batch/rank/step ranges)
NVTX = os.environ.get("PACKMLA_NVTX", "0") == "1"
_PROFILING = [False]  # set between /start_profile and /stop_profile: ranges are emitted then too


def nvtx_range(name: str):
    if (NVTX or _PROFILING[0]) and torch.cuda.is_available():
        return torch.cuda.nvtx.range(name)
    return contextlib.nullcontext()


@dataclass
class SamplingParams:
    max_new_tokens: int = 16
    temperature: float = 0.0  # 0 = greedy
    ignore_eos: bool = True
    eos_token_id: int | None = None
    # log-probabilities (the OpenAI completions `echo` / `logprobs`): `prompt_logprobs` = k >= 0 scores
    # every prompt token after the first (and keeps the top k at each position); `logprobs` records the
    # log-probability of each generated token.  A request scoring its prompt prefills all of it (no prefix
    # reuse); max_new_tokens = 0 then generates nothing.
    prompt_logprobs: int | None = None
    logprobs: bool = False
    # score prompt tokens from this index on (SGLang's logprob_start_len): the tokens before it may come
    # from a prefix cache, so requests sharing a long context re-prefill only their own tail
    prompt_logprobs_from: int = 0


@dataclass
class Request:
    rid: int
    prompt: list[int]
    params: SamplingParams
    output_ids: list[int] = field(default_factory=list)
    slot: int = -1
    prefilled: int = 0
    finished: bool = False
    t_arrival: float = 0.0
    t_first_token: float | None = None
    t_finish: float | None = None
    cached_tokens: int = 0  # prompt tokens whose KV came from the device prefix cache or the host tier
    block_tail: object = None  # the prefix-block node its prefill has reached (chains the next block)
    prompt_lp: list = field(default_factory=list)  # per prompt token: log-probability (None for the first)
    prompt_top: list = field(default_factory=list)  # per prompt token: [(token, log-probability)] top-k
    output_lp: list = field(default_factory=list)  # per generated token (SamplingParams.logprobs)

    @property
    def context_len(self) -> int:
        return self.prefilled + len(self.output_ids)


class DecodeGraphRunner:
    """Captures model.decode(+ sampling) per padded batch size; replays with copied inputs."""

    def __init__(self, model: V4FlashModel, buckets: list[int], dummy_slot: int, enabled: bool):
        self.model = model
        self.device = model.device
        self.buckets = sorted(buckets)
        self.max_b = self.buckets[-1]
        self.dummy_slot = dummy_slot
        self.enabled = enabled and self.device.type == "cuda"
        dev = self.device
        self.tokens = torch.zeros(self.max_b, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(self.max_b, dtype=torch.int64, device=dev)
        self.slots = torch.full((self.max_b,), dummy_slot, dtype=torch.int64, device=dev)
        self.temps = torch.zeros(self.max_b, dtype=torch.float32, device=dev)
        self.out_tokens = torch.zeros(self.max_b, dtype=torch.int64, device=dev)
        self.out_lp = torch.zeros(self.max_b, dtype=torch.float32, device=dev)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.pool_handle = None

    def _forward(self, b: int) -> None:
        if self.model.dp:  # every rank runs the same padded batch in a DP decode step
            self.model.dp_counts = [b] * self.model.world
        logits = self.model.decode(self.tokens[:b], self.positions[:b], self.slots[:b])
        self.out_tokens[:b] = sample(logits, self.temps[:b])
        self.out_lp[:b] = logits.gather(1, self.out_tokens[:b, None])[:, 0] - torch.logsumexp(logits, -1)

    def bucket(self, b: int) -> int:
        for s in self.buckets:
            if s >= b:
                return s
        raise ValueError(f"batch {b} exceeds the largest graph bucket {self.max_b}")

    def capture(self, sizes: list[int] | None = None) -> None:
        if not self.enabled:
            return
        sizes = sizes or self.buckets
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for b in sorted(sizes, reverse=True):
                self.slots[:b] = self.dummy_slot
                self.positions[:b] = 0
                self._forward(b)  # warm-up (allocations, lazy inits)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=self.pool_handle, stream=stream):
                    self._forward(b)
                if self.pool_handle is None:
                    self.pool_handle = g.pool()
                self.graphs[b] = g
        torch.cuda.current_stream(self.device).wait_stream(stream)
        self.model.pool.comp_state_reset(self.dummy_slot)

    def run(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, temps: torch.Tensor,
            pad_to: int = 0) -> torch.Tensor:
        """Inputs are (pinned) host or device tensors of length b; returns device token ids [b].  The batch
        runs padded to at least `pad_to` rows (DP attention: the batch every rank runs)."""
        b = tokens.shape[0]
        bp = self.bucket(max(b, pad_to)) if self.enabled else max(b, pad_to)
        self.tokens[:b].copy_(tokens, non_blocking=True)
        self.positions[:b].copy_(positions, non_blocking=True)
        self.slots[:b].copy_(slots, non_blocking=True)
        self.temps[:b].copy_(temps, non_blocking=True)
        if bp > b:
            self.slots[b:bp] = self.dummy_slot
            self.positions[b:bp] = 0
            self.tokens[b:bp] = 0
        with nvtx_range(f"decode.{'graph' if self.enabled and bp in self.graphs else 'eager'} b={b} padded={bp}"):
            if self.enabled and bp in self.graphs:
                self.graphs[bp].replay()
            else:
                self._forward(bp)
        return self.out_tokens[:b]

    def release(self) -> None:
        """Destroy the captured graphs (they hold NCCL calls under TP: release before destroying the group)."""
        for g in self.graphs.values():
            g.reset()
        self.graphs.clear()
        self.pool_handle = None


def sample(logits: torch.Tensor, temps: torch.Tensor) -> torch.Tensor:
    """Greedy where temperature == 0, else Gumbel-max sampling (graph-capturable)."""
    greedy = logits.argmax(-1)
    u = torch.rand_like(logits).clamp_(min=1e-20)
    g = -torch.log(-torch.log(u))
    t = temps.clamp(min=1e-5)[:, None]
    sampled = (logits / t + g).argmax(-1)
    return torch.where(temps > 0, sampled, greedy)


class Engine:
    def __init__(self, model_cfg: ModelConfig, engine_cfg: EngineConfig, model: V4FlashModel, pool: KVPool,
                 comm=None):
        self.cfg = model_cfg
        self.ecfg = engine_cfg
        self.model = model
        self.pool = pool
        self.comm = comm
        self.device = pool.device
        self.metrics = Metrics()
        self.dp = bool(engine_cfg.dp_attention) and getattr(comm, "world", 1) > 1
        self.rank = getattr(comm, "rank", 0)
        self.world = getattr(comm, "world", 1)
        self._owner: dict[int, int] = {}  # DP attention: owners other than rid % world (forked choices)
        self.dummy_slot = pool.max_requests - 1
        pool._free_slots.remove(self.dummy_slot)
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.done: dict[int, Request] = {}
        self._ids = itertools.count()
        buckets = [b for b in engine_cfg.cuda_graph_bs if b <= pool.max_requests - 1] or [1]
        self.runner = DecodeGraphRunner(model, buckets, self.dummy_slot, not engine_cfg.disable_cuda_graph)
        pin = self.device.type == "cuda"
        mb = self.runner.max_b
        self._h_tokens = torch.zeros(mb, dtype=torch.int64, pin_memory=pin)
        self._h_pos = torch.zeros(mb, dtype=torch.int64, pin_memory=pin)
        self._h_slots = torch.zeros(mb, dtype=torch.int64, pin_memory=pin)
        self._h_temps = torch.zeros(mb, dtype=torch.float32, pin_memory=pin)
        self._h_out = torch.zeros(mb, dtype=torch.int64, pin_memory=pin)
        self._h_lp = torch.zeros(mb, dtype=torch.float32, pin_memory=pin)
        self.h2d_bytes_last = 0
        self.d2h_bytes_last = 0
        self._last_prefill = False
        # optional device timing of steps: when set to a list, every step appends ("prefill" | "decode",
        # start event, end event) recorded on the current stream around its device work
        self.step_events: list | None = None
        # device prefix cache: processed tokens of a finished request -> its retained slot (LRU order)
        self.retained: OrderedDict[tuple, int] = OrderedDict()
        # prompt forks: leader rid -> requests with the same prompt that copy its KV once it is prefilled
        self.forks: dict[int, list[Request]] = {}
        self.blocks = None
        if (engine_cfg.prefix_cache and engine_cfg.prefix_block_tokens
                and engine_cfg.prefix_block_tokens % engine_cfg.chunked_prefill_size == 0):
            from ..kv.prefix_blocks import PrefixBlockCache

            self.blocks = PrefixBlockCache(pool, engine_cfg.prefix_block_tokens)
        self.hicache = None
        if engine_cfg.enable_hierarchical_cache:
            from ..kv.hicache import HostKVCache

            self.hicache = HostKVCache(pool, engine_cfg.hicache_ratio, engine_cfg.hicache_mem_layout)
            if self.blocks is not None:
                self.blocks.host = self.hicache  # evicted prompt blocks move to the host tier

    # ------------------------------------------------------------------ construction
    @classmethod
    def build(cls, model_cfg: ModelConfig, engine_cfg: EngineConfig, device="cuda", rank: int = 0, world: int = 1,
              comm=None, max_context: int = 1 << 15, max_requests: int | None = None, kv_bytes: int | None = None,
              seed: int = 0, weights: dict | None = None) -> "Engine":
        engine_cfg.validate()
        dev = torch.device(device)
        W = weights if weights is not None else init_weights(model_cfg, rank, world, dev, seed,
                                                             dp_attention=engine_cfg.dp_attention)
        if dev.type == "cuda" and model_cfg.expert_format == "mxfp4":
            from ..ops.moe import prepare_experts, prepare_experts_mx

            prep = prepare_experts if engine_cfg.moe_precision == "bf16" else prepare_experts_mx
            for lw in W["layers"]:  # one-time kernel layout of the experts (canonical copies dropped)
                prep(lw, drop_canonical=weights is None)
        max_requests = max_requests or engine_cfg.max_running_requests
        max_requests += 1  # + dummy slot for padded graph rows
        if kv_bytes is None:
            if dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(dev)
                kv_bytes = int(free * engine_cfg.mem_fraction_static) - (2 << 30)
            else:
                kv_bytes = 64 << 20
        cap = plan_capacity(model_cfg, engine_cfg, kv_bytes)
        pages = max(cap.num_pages, 1)
        pool = KVPool(model_cfg, engine_cfg, pages, max_requests, max_context, dev)
        model = V4FlashModel(model_cfg, W, pool, comm)
        model.moe_precision = engine_cfg.moe_precision
        eng = cls(model_cfg, engine_cfg, model, pool, comm)
        eng.capacity = cap
        return eng

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt: list[int], params: SamplingParams | None = None) -> int:
        if not prompt:
            raise ValueError("empty prompt")
        req = Request(next(self._ids), list(prompt), params or SamplingParams(), t_arrival=time.perf_counter())
        if not self.owns(req.rid):  # DP attention: another rank serves it
            return req.rid
        self.waiting.append(req)
        self.metrics.inc("requests_received")
        return req.rid

    def add_group(self, prompt: list[int], params: SamplingParams | None = None, n: int = 1) -> list[int]:
        """`n` requests with one prompt (the OpenAI `n`): the first is prefilled, the others copy its KV
        when its prefill ends and sample their own first token from the same logits, so the prompt is
        prefilled once.  A copy that finds no free slot or pages then is prefilled on its own later."""
        lead = self.add_request(prompt, params)
        if n <= 1:
            return [lead]
        followers = [Request(next(self._ids), list(prompt), params or SamplingParams(), t_arrival=time.perf_counter())
                     for _ in range(n - 1)]
        if self.dp:  # the copies live where the leader's KV is
            for f in followers:
                self._owner[f.rid] = lead % self.world
            if not self.owns(lead):
                return [lead] + [f.rid for f in followers]
        self.forks[lead] = followers
        self.metrics.inc("requests_received", n - 1)
        return [lead] + [f.rid for f in followers]

    def _fork(self, leader: Request, logits: torch.Tensor) -> list[tuple[int, int]]:
        """Start the followers of `leader` (just prefilled, slot intact) from copies of its KV."""
        produced = []
        n = len(leader.prompt)
        for f in self.forks.pop(leader.rid, []):
            need = n + f.params.max_new_tokens
            pages = (need + KVPool.TOKENS_PER_PAGE - 1) // KVPool.TOKENS_PER_PAGE
            c128 = (need + KVPool.TOKENS_PER_C128_PAGE - 1) // KVPool.TOKENS_PER_C128_PAGE
            while ((not self.pool._free_slots or pages > self.pool.pages.free or c128 > self.pool.c128_pages.free)
                   and self._evict_cached()):
                pass
            if (len(self.running) + 1 >= self.runner.max_b or not self.pool._free_slots
                    or pages > self.pool.pages.free or c128 > self.pool.c128_pages.free):
                self.waiting.append(f)  # no room now: an ordinary prefill later
                continue
            f.slot = self.pool.admit(need)
            self.pool.clone_kv(leader.slot, f.slot, n)
            f.prefilled = f.cached_tokens = n
            self.metrics.inc("fork_copied_tokens", n)
            temp = torch.tensor([f.params.temperature], device=self.device)
            tok = int(sample(logits[None], temp)[0])
            self._emit(f, tok)
            if not f.finished:
                self.running.append(f)
            produced.append((f.rid, tok))
        return produced

    def owns(self, rid: int) -> bool:
        """Whether this rank serves request rid (always, unless DP attention spreads the requests)."""
        return not self.dp or self._owner.get(rid, rid % self.world) == self.rank

    def has_work(self) -> bool:
        if self.dp:  # any rank's work keeps every rank stepping (the MoE exchanges need all of them)
            local = int(bool(self.waiting or self.running))
            return any(v[0] for v in self.comm.exchange_ints([local], self.device))
        return bool(self.waiting or self.running or self.forks)

    def result(self, rid: int) -> Request:
        if not self.owns(rid):
            raise KeyError(f"request {rid} is served by rank {self._owner.get(rid, rid % self.world)}")
        return self.done[rid]

    def abort(self, rid: int) -> bool:
        followers = self.forks.pop(rid, None)
        if followers:  # the copies of an aborted leader are prefilled on their own
            self.waiting.extend(followers)
        for lead, fs in list(self.forks.items()):
            for f in fs:
                if f.rid == rid:
                    fs.remove(f)
                    f.finished = True
                    self.done[rid] = f
                    self.metrics.inc("requests_aborted")
                    return True
        for q in (self.waiting, self.running):
            for r in list(q):
                if r.rid == rid:
                    q.remove(r)
                    if r.slot >= 0:
                        self.pool.release(r.slot)
                    r.finished = True
                    self.done[rid] = r
                    self.metrics.inc("requests_aborted")
                    return True
        return False

    # ------------------------------------------------------------------ scheduling
    # ------------------------------------------------------------------ device prefix cache
    def _retain(self, req: Request) -> None:
        """Keep a finished request's slot: its KV covers every token but the last output."""
        key = tuple(req.prompt + req.output_ids[:-1])
        old = self.retained.pop(key, None)
        if old is not None:
            self.pool.release(old)
        self.retained[key] = req.slot

    def _evict_retained(self) -> bool:
        """Release the least recently used retained slot; False when none is left."""
        if not self.retained:
            return False
        _, slot = self.retained.popitem(last=False)
        self.pool.release(slot)
        self.metrics.inc("prefix_cache_evictions")
        return True

    def _evict_cached(self) -> bool:
        """Free cached KV for admission: a retained slot first, else the least recently used prefix block."""
        if self._evict_retained():
            return True
        if self.blocks is not None and self.blocks.evict_one():
            self.metrics.inc("prefix_block_evictions")
            return True
        return False

    def _match_retained(self, prompt: list[int], limit: int | None = None) -> tuple | None:
        """Longest retained context that is a strict prefix of `prompt` (at least one token to prefill),
        at most `limit` tokens long."""
        best = None
        limit = len(prompt) - 1 if limit is None else min(limit, len(prompt) - 1)
        for key in self.retained:
            if len(key) <= limit and (best is None or len(key) > len(best)) and tuple(prompt[:len(key)]) == key:
                best = key
        return best

    def flush_prefix_cache(self) -> None:
        while self._evict_retained():
            pass
        if self.blocks is not None:
            self.blocks.flush()

    def _adopt(self, req: Request, need: int, limit: int | None = None) -> bool | None:
        """Continue `req` in the retained slot of its longest cached prefix, growing its pages.
        True: adopted; False: no cached prefix; None: cached, but the pages do not fit yet (a full
        admission would need more, so the request waits for running requests to finish)."""
        key = self._match_retained(req.prompt, limit)
        if key is None:
            return False
        slot = self.retained.pop(key)
        grow = ((need + KVPool.TOKENS_PER_PAGE - 1) // KVPool.TOKENS_PER_PAGE
                - len(self.pool._req_pages[slot]))
        grow128 = ((need + KVPool.TOKENS_PER_C128_PAGE - 1) // KVPool.TOKENS_PER_C128_PAGE
                   - len(self.pool._req_c128[slot]))
        while (grow > self.pool.pages.free or grow128 > self.pool.c128_pages.free) and self._evict_cached():
            pass
        if grow > self.pool.pages.free or grow128 > self.pool.c128_pages.free:
            self.retained[key] = slot  # keep it for later; admission waits for running requests to finish
            return None
        self.pool.ensure(slot, need)
        req.slot, req.prefilled = slot, len(key)
        req.cached_tokens = len(key)
        self.metrics.inc("prefix_cache_hit_tokens", len(key))
        return True

    def _admit(self) -> Request | None:
        if not self.waiting:
            return None
        req = self.waiting[0]
        if req.slot < 0:
            need = len(req.prompt) + req.params.max_new_tokens
            if need > self.pool.max_context:
                self.waiting.popleft()
                raise ValueError(f"request {req.rid} needs {need} tokens > max_context {self.pool.max_context}")
            if len(self.running) >= self.runner.max_b:
                return None
            # a scored prompt reuses cached KV only before its first scored token's predecessor
            reuse_limit = (len(req.prompt) if req.params.prompt_logprobs is None
                           else max(0, req.params.prompt_logprobs_from - 1))
            reuse = reuse_limit > 0
            if self.retained and reuse:
                adopted = self._adopt(req, need, reuse_limit)
                if adopted is None:
                    return None
                if adopted:
                    return req
            # shared prompt blocks: their pages are mapped, not allocated (pinned against eviction meanwhile);
            # host-resident ones are copied back into new pages first
            chain = self.blocks.match(req.prompt) if self.blocks is not None and reuse else []
            while chain and (chain[-1].index + 1) * self.blocks.block > reuse_limit:
                chain.pop()
            n_shared, n_shared128 = self.blocks.shared_counts(chain) if chain else (0, 0)
            r_pages, r_c128 = self.blocks.restore_need(chain) if chain else (0, 0)
            for n in chain:
                n.pins += 1
            pages_needed = (need + KVPool.TOKENS_PER_PAGE - 1) // KVPool.TOKENS_PER_PAGE - n_shared + r_pages
            c128_needed = ((need + KVPool.TOKENS_PER_C128_PAGE - 1) // KVPool.TOKENS_PER_C128_PAGE
                           - n_shared128 + r_c128)
            while ((not self.pool._free_slots or pages_needed > self.pool.pages.free
                    or c128_needed > self.pool.c128_pages.free) and self._evict_cached()):
                pass
            fits = not (not self.pool._free_slots or pages_needed > self.pool.pages.free
                        or c128_needed > self.pool.c128_pages.free)
            if fits:
                if r_pages:
                    self.metrics.inc("prefix_block_host_hits", self.blocks.promote(chain))
                shared, shared128 = self.blocks.shared_pages(chain) if chain else ([], [])
                req.slot = self.pool.admit(need, shared, shared128)  # the request's own page references
            for n in chain:
                n.pins -= 1
            if not fits:
                return None
            if chain:  # resume at the end of the last shared block
                self.blocks.attach(chain, req.slot)
                req.prefilled = req.cached_tokens = (chain[-1].index + 1) * self.blocks.block
                req.block_tail = chain[-1]
                self.metrics.inc("prefix_block_hit_tokens", req.prefilled)
            elif self.hicache is not None and req.params.prompt_logprobs is None:
                entry = self.hicache.match(req.prompt)
                if entry is not None:  # earlier turn of this context: restore its KV, prefill the rest
                    req.prefilled = self.hicache.restore(entry, req.slot)
                    req.cached_tokens = req.prefilled
                    self.metrics.inc("hicache_hit_tokens", req.prefilled)
        return req

    def step(self) -> list[tuple[int, int]]:
        """Run one prefill chunk (if a request is waiting and fits) or one decode step; when both are
        pending they alternate (`EngineConfig.prefill_decode_interleave`).

        Returns the (rid, token) pairs produced by this step.
        """
        rank = getattr(self.comm, "rank", 0)
        if self.dp:
            return self._step_dp()
        # with both kinds of work pending, prefill chunks and decode steps alternate: a queue of long
        # prompts must not stall the running requests' token streams for many steps
        if self.running and self._last_prefill and self.ecfg.prefill_decode_interleave:
            self._last_prefill = False
            with nvtx_range(f"scheduler.batch rank={rank} decode b={len(self.running)}"):
                return self._decode()
        req = self._admit()
        if req is not None:
            self._last_prefill = True
            with nvtx_range(f"scheduler.batch rank={rank} prefill rid={req.rid} start={req.prefilled}"):
                return self._prefill_chunk(req)
        if self.running:
            self._last_prefill = False
            with nvtx_range(f"scheduler.batch rank={rank} decode b={len(self.running)}"):
                return self._decode()
        return []

    def _step_dp(self) -> list[tuple[int, int]]:
        """One DP-attention step.  Every rank proposes (tokens of its next prefill chunk, running requests);
        the step is a decode step when any rank has running requests and either the last step was a
        prefill (interleaving) or no rank can prefill; otherwise a prefill step, in which ranks without a
        chunk run a token-less forward.  Decode steps pad every rank to the same batch bucket."""
        req = self._admit()
        p_tok = min(self.ecfg.chunked_prefill_size, len(req.prompt) - req.prefilled) if req is not None else 0
        plans = self.comm.exchange_ints([p_tok, len(self.running)], self.device)
        any_prefill = any(p[0] for p in plans)
        max_run = max(p[1] for p in plans)
        if max_run and (not any_prefill or (self._last_prefill and self.ecfg.prefill_decode_interleave)):
            self._last_prefill = False
            with nvtx_range(f"scheduler.batch rank={self.rank} dp-decode b={len(self.running)} pad={max_run}"):
                return self._decode(pad_to=max_run)
        if not any_prefill:
            return []
        self._last_prefill = True
        self.model.dp_counts = [p[0] for p in plans]
        if req is not None:
            with nvtx_range(f"scheduler.batch rank={self.rank} dp-prefill rid={req.rid} start={req.prefilled}"):
                return self._prefill_chunk(req)
        ev = self._events("prefill")
        if ev is not None:
            ev[0].record()
        self.model.dp_idle_forward()
        if ev is not None:
            ev[1].record()
        return []

    def _events(self, kind: str):
        """(start, end) CUDA events of this step when step timing is on, else None."""
        if self.step_events is None or self.device.type != "cuda":
            return None
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self.step_events.append((kind, ev[0], ev[1]))
        return ev

    def _prefill_chunk(self, req: Request) -> list[tuple[int, int]]:
        chunk = self.ecfg.chunked_prefill_size
        start = req.prefilled
        toks = req.prompt[start:start + chunk]
        t = torch.tensor(toks, dtype=torch.int64)
        ev = self._events("prefill")
        if ev is not None:
            ev[0].record()
        if self.device.type == "cuda":
            t = t.pin_memory().to(self.device, non_blocking=True)
        self.h2d_bytes_last = t.numel() * t.element_size()
        k = req.params.prompt_logprobs
        if k is None:
            logits = self.model.prefill(t, start, req.slot)
        else:  # score the next prompt token after the chunk's positions from the scoring start on
            if not req.prompt_lp:  # tokens before the first scored one (a reused prefix included): None
                n0 = max(1, req.params.prompt_logprobs_from, start + 1)
                req.prompt_lp.extend([None] * n0)
                req.prompt_top.extend([None] * n0)
            first = len(req.prompt_lp) - 1 - start  # chunk row predicting the next unscored token
            targets = torch.tensor(req.prompt[start + first + 1:start + len(toks) + 1], dtype=torch.int64,
                                   device=self.device)
            if first >= 0 and targets.numel():
                logits, (lp, tv, ti) = self.model.prefill(t, start, req.slot, score=(targets, k, first))
                req.prompt_lp.extend(lp.tolist())
                req.prompt_top.extend([list(zip(i, v)) for i, v in zip(ti.tolist(), tv.tolist())])
            else:
                logits = self.model.prefill(t, start, req.slot)
        if ev is not None:
            ev[1].record()
        req.prefilled += len(toks)
        self.metrics.inc("prefill_tokens", len(toks))
        if self.blocks is not None and req.prefilled % self.blocks.block == 0:
            # the chunk ended on a block boundary: cache the block if it extends the request's cached chain
            idx, tail = req.prefilled // self.blocks.block - 1, req.block_tail
            if (tail is None and idx == 0) or (tail is not None and tail.index == idx - 1):
                req.block_tail = self.blocks.insert(req.prompt, req.slot, idx, tail)
        if req.prefilled < len(req.prompt):
            return []
        self.waiting.popleft()
        if req.params.max_new_tokens == 0:  # prompt scoring only
            req.t_first_token = time.perf_counter()
            self._finish(req)
            return [(req.rid, None)]
        temp = torch.tensor([req.params.temperature], device=self.device)
        tok = int(sample(logits[None], temp)[0])
        if req.params.logprobs:
            req.output_lp.append(float(logits[tok] - torch.logsumexp(logits, -1)))
        forked = self._fork(req, logits) if req.rid in self.forks else []  # before the leader can finish
        self._emit(req, tok)
        if not req.finished:
            self.running.append(req)
        return [(req.rid, tok)] + forked

    def _decode(self, pad_to: int = 0) -> list[tuple[int, int]]:
        reqs = self.running
        b = len(reqs)
        for i, r in enumerate(reqs):
            self._h_tokens[i] = r.output_ids[-1]
            self._h_pos[i] = r.context_len - 1
            self._h_slots[i] = r.slot
            self._h_temps[i] = r.params.temperature
        self.h2d_bytes_last = b * (8 + 8 + 8 + 4)
        ev = self._events("decode")
        if ev is not None:
            ev[0].record()
        out = self.runner.run(self._h_tokens[:b], self._h_pos[:b], self._h_slots[:b], self._h_temps[:b], pad_to)
        self._h_out[:b].copy_(out, non_blocking=True)
        want_lp = any(r.params.logprobs for r in reqs)
        if want_lp:
            self._h_lp[:b].copy_(self.runner.out_lp[:b], non_blocking=True)
        if ev is not None:
            ev[1].record()
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        self.d2h_bytes_last = b * 8
        toks = self._h_out[:b].tolist()
        lps = self._h_lp[:b].tolist() if want_lp else [None] * b
        produced = []
        for r, tok, lp in zip(list(reqs), toks, lps):
            if r.params.logprobs:
                r.output_lp.append(lp)
            self._emit(r, tok)
            produced.append((r.rid, tok))
        self.running = [r for r in reqs if not r.finished]
        if b:
            self.metrics.inc("decode_steps")
            self.metrics.inc("decode_tokens", b)
        return produced

    def _emit(self, req: Request, tok: int) -> None:
        if req.t_first_token is None:
            req.t_first_token = time.perf_counter()
        req.output_ids.append(tok)
        eos = req.params.eos_token_id
        if len(req.output_ids) >= req.params.max_new_tokens or (not req.params.ignore_eos and eos is not None
                                                                 and tok == eos):
            self._finish(req)

    def _finish(self, req: Request) -> None:
        req.finished = True
        req.t_finish = time.perf_counter()
        if self.hicache is not None:  # write through: every token but the last has its KV stored
            self.hicache.save(req.slot, req.prompt + req.output_ids[:-1])
        if self.ecfg.prefix_cache:
            self._retain(req)
        else:
            self.pool.release(req.slot)
        self.done[req.rid] = req
        self.metrics.inc("requests_finished")

    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None) -> list[list[int]]:
        rids = [self.add_request(p, params) for p in prompts]
        while self.has_work():
            self.step()
        return [self.result(r).output_ids for r in rids]

    def profile(self, on: bool) -> bool:
        """Open (on) or close the CUDA profiler capture range (cudaProfilerStart / Stop), which Nsight
        Systems / Compute honour with `--capture-range=cudaProfilerApi`, and emit NVTX ranges while it is
        open (reference: SGLang's /start_profile, /stop_profile).  Returns whether the state changed."""
        if on == _PROFILING[0]:
            return False
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            (torch.cuda.profiler.start if on else torch.cuda.profiler.stop)()
        _PROFILING[0] = on
        self.metrics.inc("profile_ranges_opened" if on else "profile_ranges_closed")
        return True

    def flush_cache(self) -> None:
        """Drop cached KV of finished requests (device prefix cache and the HiCache host tier)."""
        self.flush_prefix_cache()
        if self.hicache is not None:
            self.hicache.flush()

    def server_info(self) -> dict:
        return {
            "kv_cache_format": self.ecfg.kv_cache_format,
            "max_total_num_tokens": self.capacity.max_total_tokens,
            "bytes_per_full_token": self.capacity.bytes_per_full_token,
            "num_pages": self.pool.num_pages,
            "context_length": self.pool.max_context,
            "max_running_requests": self.pool.max_requests - 1,
            "cuda_graph_bs": self.runner.buckets,
            "tp": self.ecfg.tp,
            "prefix_cache": self.ecfg.prefix_cache,
            "prefix_cache_retained": len(self.retained),
            "prefix_blocks": len(self.blocks.nodes) if self.blocks is not None else 0,
            "prefix_blocks_on_host": self.blocks.host_nodes if self.blocks is not None else 0,
            "enable_hierarchical_cache": self.hicache is not None,
            "hicache_host_bytes": self.hicache.host_bytes() if self.hicache is not None else 0,
        }

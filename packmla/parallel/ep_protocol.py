"""Executable model of a fused expert-parallel exchange over symmetric peer buffers (dispatch, local
experts, combine), for checking its buffer reuse and progress on the host before a kernel implements it.

Reference behaviour: DeepEP dispatch / combine under `--ep` (scripts/local/run-server.sh:89-100): each
(token, expert) pair goes to the expert's owner and comes back weighted.  `packmla.parallel.ep.EPMoE`
does it with two NCCL all-to-alls; the fused form replaces them with stores into peers' buffers:

* every rank r owns, in its symmetric memory, one receive region per source s (`rows[r][s][i]`, capacity
  T k pairs, so a sender needs no offsets from other senders) and one return region per destination d
  (`back[r][d][i]`);
* dispatch (rank s, call c): pair j of s's routing, owned by d, is the i-th pair s sends to d; s stores
  the row into rows[d][s][i], then its count and `flag_rows[d][s] = c` (release);
* each owner d acquires `flag_rows[d][s] >= c` for every s, runs its experts on the received rows and
  stores output i into back[s][d][i], then releases `flag_back[s][d] = c`;
* source s acquires `flag_back[s][d] >= c` for every d and sums its pairs in routing order.

One buffer per region suffices: s writes call c + 1 rows into d's region only after it has received all
of d's call-c outputs, and d sends those only after it has read s's call-c rows.  The same argument covers
the return regions.  `wait_all_back=False` lets a source start the next dispatch after one owner's return
(a bug the checker must catch as a stale read).  Memory is modelled sequentially consistent at step
granularity, with flags compared `>= c`, as in `packmla.parallel.protocol`.
"""
from __future__ import annotations

import random

from .protocol import ProtocolError


class EPExchangeModel:
    def __init__(self, world: int, tokens: int, topk: int, experts: int, calls: int, seed: int = 0,
                 wait_all_back: bool = True, arrival_order: bool = False):
        """`arrival_order`: an owner serves the sources in the order their flags arrive (any released source
        next), as a kernel that overlaps the exchange with the expert GEMMs would, instead of 0, 1, ..."""
        if experts % world:
            raise ValueError("experts must divide evenly over the ranks")
        rng = random.Random(seed)
        self.world, self.T, self.k, self.E, self.calls = world, tokens, topk, experts, calls
        self.local = experts // world
        self.wait_all_back = wait_all_back
        self.arrival_order = arrival_order
        self.served: dict = {}
        self._rng = random.Random(seed)
        # routing[c][r] = list of (token, expert) pairs of rank r in routing order
        self.routing = [[[(t, rng.randrange(experts)) for t in range(tokens) for _ in range(topk)]
                         for _ in range(world)] for _ in range(calls)]
        W = range(world)
        self.rows = {(d, s): {} for d in W for s in W}     # rows[d][s][i] = tag
        self.back = {(s, d): {} for s in W for d in W}     # back[s][d][i] = tag
        self.flag_rows = {(d, s): 0 for d in W for s in W}
        self.flag_back = {(s, d): 0 for s in W for d in W}
        self.count = {(d, s): 0 for d in W for s in W}
        self.results: dict = {}
        self.progs = [self._program(r) for r in W]
        self.pcs = [0] * world

    # tags: a dispatched row = ("row", call, src, pair); a returned output = ("out", call, src, pair)
    def _program(self, r: int) -> list:
        steps = []
        for c in range(1, self.calls + 1):
            pairs = self.routing[c - 1][r]
            per_dest: dict[int, list[int]] = {}
            for j, (_, e) in enumerate(pairs):
                per_dest.setdefault(e // self.local, []).append(j)
            for d in range(self.world):  # dispatch: rows, then count and flag
                for i, j in enumerate(per_dest.get(d, [])):
                    steps.append(("store_row", c, d, i, j))
                steps.append(("release_rows", c, d, len(per_dest.get(d, []))))
            for s in range(self.world):  # owner side: wait for every source, compute, return
                if self.arrival_order:
                    steps.append(("serve_any", c))
                else:
                    steps.append(("acquire_rows", c, s))
                    steps.append(("compute_return", c, s))
            waits = range(self.world) if self.wait_all_back else [r]
            for d in waits:
                steps.append(("acquire_back", c, d))
            steps.append(("combine", c, dict(per_dest)))
        return steps

    def _enabled(self, r: int) -> bool:
        if self.pcs[r] >= len(self.progs[r]):
            return False
        op = self.progs[r][self.pcs[r]]
        if op[0] == "acquire_rows":
            return self.flag_rows[(r, op[2])] >= op[1]
        if op[0] == "acquire_back":
            return self.flag_back[(r, op[2])] >= op[1]
        if op[0] == "serve_any":
            return bool(self._ready_sources(r, op[1]))
        return True

    def _ready_sources(self, r: int, c: int) -> list[int]:
        done = self.served.setdefault((r, c), set())
        return [s for s in range(self.world) if s not in done and self.flag_rows[(r, s)] >= c]

    def _serve(self, r: int, c: int, s: int) -> None:
        n = self.count[(r, s)]
        for i in range(n):
            tag = self.rows[(r, s)].get(i)
            if tag is None or tag[0] != "row" or tag[1] != c or tag[2] != s:
                raise ProtocolError(f"rank {r} read {tag} for call {c} row {i} from rank {s}")
            self.back[(s, r)][i] = ("out", c, s, tag[3])
        self.flag_back[(s, r)] = c

    def _step(self, r: int) -> None:
        op = self.progs[r][self.pcs[r]]
        kind, c = op[0], op[1]
        if kind == "store_row":
            _, _, d, i, j = op
            self.rows[(d, r)][i] = ("row", c, r, j)
        elif kind == "release_rows":
            _, _, d, n = op
            self.count[(d, r)] = n
            self.flag_rows[(d, r)] = c
        elif kind == "compute_return":
            self._serve(r, c, op[2])
        elif kind == "serve_any":
            s = self._rng.choice(self._ready_sources(r, c))
            self.served[(r, c)].add(s)
            self._serve(r, c, s)
        elif kind == "combine":
            per_dest = op[2]
            got = {}
            for d, js in per_dest.items():
                for i, j in enumerate(js):
                    tag = self.back[(r, d)].get(i)
                    if tag != ("out", c, r, j):
                        raise ProtocolError(f"rank {r} combined {tag} for call {c} pair {j} from rank {d}")
                    got[j] = tag
            self.results[(r, c)] = sorted(got)
        self.pcs[r] += 1

    def run(self, rng: random.Random) -> None:
        while True:
            ready = [r for r in range(self.world) if self._enabled(r)]
            if not ready:
                if any(self.pcs[r] < len(self.progs[r]) for r in range(self.world)):
                    raise ProtocolError("deadlock: unfinished ranks and no enabled step")
                break
            self._step(rng.choice(ready))
        for r in range(self.world):
            for c in range(1, self.calls + 1):
                if self.results.get((r, c)) != list(range(self.T * self.k)):
                    raise ProtocolError(f"rank {r} call {c} combined {self.results.get((r, c))}")


def explore(world: int, tokens: int, topk: int, experts: int, calls: int, schedules: int, seed: int = 0,
            wait_all_back: bool = True, arrival_order: bool = False) -> int:
    """Run `schedules` random interleavings; returns how many completed (raises on the first race)."""
    rng = random.Random(seed)
    for n in range(schedules):
        EPExchangeModel(world, tokens, topk, experts, calls, seed=seed + n, wait_all_back=wait_all_back,
                        arrival_order=arrival_order).run(rng)
    return schedules


def emulate_exchange(h: list, ids: list, w: list, experts: int, expert_fn) -> list:
    """The data path of the protocol above on tensors, all ranks in one process: the oracle a fused kernel
    is checked against.  h[r] [T, H], ids[r] / w[r] [T, k] of rank r; `expert_fn(rows, global_expert_ids)`
    returns the unweighted outputs.  Each rank's symmetric memory holds rows[r] [world, T k, H] (one
    region per source) and back[r] [world, T k, H] (one region per owner); pair j of source s that owner d
    receives as its i-th lands at rows[d][s, i] and returns to back[s][d, i].  Returns the per-rank fp32
    sums over k in routing order."""
    import torch

    world = len(h)
    T, k = ids[0].shape
    H = h[0].shape[1]
    local = experts // world
    rows = [torch.zeros(world, T * k, H, dtype=h[0].dtype) for _ in range(world)]
    rows_ids = [torch.full((world, T * k), -1, dtype=torch.int64) for _ in range(world)]
    back = [torch.zeros(world, T * k, H, dtype=torch.float32) for _ in range(world)]
    count = [[0] * world for _ in range(world)]
    index = []  # index[s][j] = (owner, slot) of pair j of source s
    for s in range(world):  # dispatch
        flat = ids[s].reshape(-1)
        slots = []
        for j in range(T * k):
            d = int(flat[j]) // local
            i = count[d][s]
            rows[d][s, i] = h[s][j // k]
            rows_ids[d][s, i] = int(flat[j])
            count[d][s] = i + 1
            slots.append((d, i))
        index.append(slots)
    for d in range(world):  # owners: experts on each source region, outputs back to the source
        for s in range(world):
            n = count[d][s]
            if n:
                back[s][d, :n] = expert_fn(rows[d][s, :n], rows_ids[d][s, :n]).float()
    out = []
    for s in range(world):  # combine in routing order
        pairs = torch.stack([back[s][d, i] for d, i in index[s]]).view(T, k, H)
        out.append((pairs * w[s].float()[..., None]).sum(1))
    return out

"""Executable model of the fused collectives' flag and slot protocol (csrc/comm_fused.cu), for race
checking on the host.

The device kernels cannot run under a race detector on this hardware pool, and 4- and 8-rank runs are
rare, so the protocol is also stated here as a program and explored under random interleavings:

* every rank makes the same sequence of calls; a call is one kernel launch of `tiles` CTAs; a rank's
  next call starts only when all CTAs of its current call have finished (stream order);
* call k of a CTA for tile t on rank r (`s = k`, the per-rank call counter):
    one-shot: store the partial into recv[d][k & 1][r][t] of every rank d, release flag_rs[d][r][t] = k,
      acquire flag_rs[r][src][t] >= k for every src, read recv[r][k & 1][src][t] for every src;
    two-shot: store the partial into recv[o][k & 1][r][t] of the tile owner o = t % world and release
      flag_rs[o][r][t] = k; the owner acquires all flags, reads all partials, stores the result into
      gath[d][t] of every rank d and releases flag_ag[d][t] = k; every rank acquires flag_ag[r][t] >= k
      and reads gath[r][t];
* flags are compared with `>= k`, as the kernels compare the wrapped difference.

Memory is modelled sequentially consistent at the granularity of these steps (the kernels order
stores before flags with system-scope release / acquire), so the model checks slot reuse, flag
monotonicity and progress, not the memory model itself.  A read that sees another call's data is a
race; a state with unfinished CTAs and no enabled step is a deadlock.  `parity_slots=False` removes
the alternation of the partial slots: the checker must then find the race in one-shot mode.
"""
from __future__ import annotations

import random
from dataclasses import dataclass


class ProtocolError(AssertionError):
    pass


@dataclass
class _Cta:
    rank: int
    tile: int
    call: int
    one_shot: bool
    steps: list
    pc: int = 0


class ProtocolModel:
    def __init__(self, world: int, tiles: int, modes: list[bool], parity_slots: bool = True,
                 rotate_owners: bool = False):
        """`modes[k]` is True for a one-shot call k (the same on every rank, as the host picks it from the
        message size).  `rotate_owners` moves each tile's two-shot owner from call to call, as happens
        when a GEMM + all-reduce call (slices owned by slice % world) follows a flat all-reduce call
        (chunks owned by chunk % world) over the same gather buffer."""
        self.world, self.tiles, self.modes, self.parity = world, tiles, list(modes), parity_slots
        self.rotate = rotate_owners
        W = range(world)
        self.recv = {(d, p, src, t): None for d in W for p in (0, 1) for src in W for t in range(tiles)}
        self.gath = {(d, t): None for d in W for t in range(tiles)}
        self.flag_rs = {(d, src, t): 0 for d in W for src in W for t in range(tiles)}
        self.flag_ag = {(d, t): 0 for d in W for t in range(tiles)}
        self.call = [0] * world          # current call index per rank (0-based into modes)
        self.active: list[list[_Cta]] = [self._launch(r, 0) for r in W]
        self.reads = 0

    # ----------------------------------------------------------------- programs
    def _slot(self, k: int) -> int:
        return (k & 1) if self.parity else 0

    def _launch(self, r: int, idx: int) -> list[_Cta]:
        if idx >= len(self.modes):
            return []
        k = idx + 1  # the call counter s starts at 1
        one = self.modes[idx]
        return [_Cta(r, t, k, one, self._program(r, t, k, one)) for t in range(self.tiles)]

    def _program(self, r: int, t: int, k: int, one_shot: bool) -> list:
        W, p = range(self.world), self._slot(k)
        owner = (t + (k if self.rotate else 0)) % self.world
        steps: list = []
        dests = list(W) if one_shot else [owner]
        steps += [("store_recv", (d, p, r, t), k) for d in dests]
        steps += [("release_rs", (d, r, t), k) for d in dests]
        if one_shot or r == owner:
            steps += [("acquire_rs", (r, src, t), k) for src in W]
            steps += [("read_recv", (r, p, src, t), k) for src in W]
        if not one_shot:
            if r == owner:
                steps += [("store_gath", (d, t), k) for d in W]
                steps += [("release_ag", (d, t), k) for d in W]
            steps += [("acquire_ag", (r, t), k), ("read_gath", (r, t), k)]
        return steps

    # ----------------------------------------------------------------- execution
    def _enabled(self, cta: _Cta) -> bool:
        op, key, k = cta.steps[cta.pc]
        if op == "acquire_rs":
            return self.flag_rs[key] >= k
        if op == "acquire_ag":
            return self.flag_ag[key] >= k
        return True

    def _apply(self, cta: _Cta) -> None:
        op, key, k = cta.steps[cta.pc]
        if op == "store_recv":
            self.recv[key] = k
        elif op == "release_rs":
            if self.flag_rs[key] > k:
                raise ProtocolError(f"flag_rs{key} moved backwards to {k}")
            self.flag_rs[key] = k
        elif op == "release_ag":
            if self.flag_ag[key] > k:
                raise ProtocolError(f"flag_ag{key} moved backwards to {k}")
            self.flag_ag[key] = k
        elif op == "store_gath":
            self.gath[key] = k
        elif op == "read_recv":
            self.reads += 1
            if self.recv[key] != k:
                raise ProtocolError(f"rank {cta.rank} tile {cta.tile} call {k} read recv{key} holding call "
                                    f"{self.recv[key]}")
        elif op == "read_gath":
            self.reads += 1
            if self.gath[key] != k:
                raise ProtocolError(f"rank {cta.rank} tile {cta.tile} call {k} read gath{key} holding call "
                                    f"{self.gath[key]}")
        cta.pc += 1

    def run(self, rng: random.Random, max_steps: int = 1_000_000) -> int:
        """Run to completion under the random schedule; returns the number of steps taken."""
        for n in range(max_steps):
            runnable = [c for ctas in self.active for c in ctas if c.pc < len(c.steps) and self._enabled(c)]
            if not runnable:
                if any(c.pc < len(c.steps) for ctas in self.active for c in ctas):
                    raise ProtocolError("deadlock: unfinished CTAs and no enabled step")
                return n
            self._apply(rng.choice(runnable))
            for r in range(self.world):  # stream order: the next launch once every CTA finished
                if self.active[r] and all(c.pc == len(c.steps) for c in self.active[r]):
                    self.call[r] += 1
                    self.active[r] = self._launch(r, self.call[r])
        raise ProtocolError("step limit reached")


def explore(world: int, tiles: int, modes: list[bool], schedules: int, seed: int = 0,
            parity_slots: bool = True, rotate_owners: bool = False) -> dict:
    """Run `schedules` random interleavings; raises ProtocolError on the first race or deadlock."""
    rng = random.Random(seed)
    steps = reads = 0
    for _ in range(schedules):
        m = ProtocolModel(world, tiles, modes, parity_slots, rotate_owners)
        steps += m.run(rng)
        reads += m.reads
    return {"world": world, "tiles": tiles, "calls": len(modes), "schedules": schedules, "steps": steps,
            "checked_reads": reads}

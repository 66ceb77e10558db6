"""Seeded synthetic multi-turn agentic traces.

A session belongs to a prefix group; its first turn is the group's system
prefix plus a random increment, and every later turn appends the previous
turn's generated tokens and a new random increment (so a turn's prompt
extends the previous turn's prompt + output, which is what the prefix cache
and the KV-aware router exploit). Token ids are uniform random; outputs are
generated with ``ignore_eos`` to the sampled length.

Presets mirror the serving configurations:

``router-plumbing`` 64 sessions x 8 turns, prefix 4096 drawn from one of 4
    seeded prefixes, increment U[128, 512], output U[32, 128], vocab 32000.
``agentic-8b``      512 sessions x 10 turns, prefix 4096 shared by groups of
    32 sessions, increment U[256, 1024], output U[128, 512], context cap
    32768, vocab 128256.
``pd-70b``          input U[8192, 32768] with 90% shared prefix reuse,
    output 256.
``ep-dsv3``         input U[2048, 16384], output U[256, 1024], vocab 129280.
``tiering-32b``     256 sessions, unique 65536-token prefix, 4 revisits,
    increment 512, output 128, vocab 151936.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field


@dataclass
class TraceSpec:
    name: str
    num_sessions: int
    turns: int
    prefix_len: int
    group_size: int            # sessions sharing one system prefix
    num_prefixes: int | None   # if set: prefixes drawn from this many seeded prefixes
    inc_range: tuple[int, int]
    out_range: tuple[int, int]
    vocab: int
    context_cap: int = 32768
    unique_prefix: bool = False


PRESETS = {
    "router-plumbing": TraceSpec("router-plumbing", 64, 8, 4096, 16, 4, (128, 512), (32, 128), 32000),
    "agentic-8b": TraceSpec("agentic-8b", 512, 10, 4096, 32, None, (256, 1024), (128, 512), 128256),
    "pd-70b": TraceSpec("pd-70b", 256, 4, 7372, 1, 8, (820, 25395), (256, 256), 128256),
    "ep-dsv3": TraceSpec("ep-dsv3", 256, 1, 0, 1, None, (2048, 16384), (256, 1024), 129280),
    "tiering-32b": TraceSpec("tiering-32b", 256, 5, 65536, 1, None, (512, 512), (128, 128), 151936, 131072, True),
    # small shape for tests
    "tiny": TraceSpec("tiny", 8, 3, 32, 4, None, (8, 16), (2, 4), 1000, 512),
}


@dataclass
class Session:
    sid: int
    group: int
    prefix: list[int]
    increments: list[list[int]]
    out_lens: list[int]
    history: list[int] = field(default_factory=list)   # prompt of the last turn + its output
    turn: int = 0
    busy: bool = False
    idle_since: float = 0.0

    def next_prompt(self) -> list[int]:
        base = self.history if self.history else self.prefix
        return base + self.increments[self.turn]

    def done(self, cap: int) -> bool:
        if self.turn >= len(self.increments):
            return True
        nxt = len(self.history or self.prefix) + len(self.increments[self.turn]) + self.out_lens[self.turn]
        return nxt > cap


def build_sessions(spec: TraceSpec, seed: int, session_ids: list[int]) -> list[Session]:
    """Sessions ``session_ids`` of the trace (a rank builds only its own)."""
    prefixes: dict[int, list[int]] = {}

    def prefix_for(group: int) -> list[int]:
        if spec.prefix_len == 0:
            return []
        key = group % spec.num_prefixes if spec.num_prefixes else group
        if key not in prefixes:
            rng = random.Random(seed * 7919 + key)
            prefixes[key] = [rng.randrange(spec.vocab) for _ in range(spec.prefix_len)]
        return prefixes[key]

    out = []
    for sid in session_ids:
        rng = random.Random(seed * 1000003 + sid)
        group = sid // max(1, spec.group_size)
        pref = prefix_for(group) if not spec.unique_prefix else [
            rng.randrange(spec.vocab) for _ in range(spec.prefix_len)]
        incs, outs = [], []
        for _ in range(spec.turns):
            n = rng.randint(*spec.inc_range)
            incs.append([rng.randrange(spec.vocab) for _ in range(n)])
            outs.append(rng.randint(*spec.out_range))
        out.append(Session(sid, group, pref, incs, outs))
    return out


def poisson_arrivals(rate: float, duration: float, seed: int, start: float = 0.0) -> list[float]:
    rng = random.Random(seed)
    t = start
    out = []
    while True:
        t += rng.expovariate(rate)
        if t >= start + duration:
            return out
        out.append(t)

"""Data-parallel attention with expert-parallel MoE (DeepSeek-V3 serving).

Every rank is a full engine over its own requests: its own scheduler, block
manager, latent KV cache and sampler, attention with all heads (DP
attention). Only the routed-expert layers are shared: each rank holds
E / world experts (``EPMoE``) and every MoE layer exchanges tokens with the
other ranks. Those exchanges are collectives, so every rank must run the
same number of forwards: each step the ranks agree over a host (gloo) group
whether any of them has work; a rank with nothing scheduled then runs a
one-token dummy forward (no cache write) to take part in the exchanges.

The router addresses the ranks as one worker with ``dp_size = world``
(rank-multiplexed targets, ``X-Data-Parallel-Rank``).

Reference counterpart: SGLang's ``--enable-dp-attention`` + ``--ep-size``
that the reference's DeepSeek recipes pass through (``infera/engine/sglang``
launcher; MoRI MoE all-to-all buffer sizing in ``__main__.py:73-100``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine


@dataclass
class EPSpec:
    rank: int
    world: int
    group: object = None      # the all-to-all process group (NCCL on GPUs, gloo on CPU)
    gloo: object = None       # host group for the lockstep vote and handle exchange
    fused: bool = False       # NVLink peer-store dispatch / return instead of NCCL all-to-all
    max_tokens: int = 256     # per-rank tokens per forward the fused buffers hold


class DPAttentionEngine:
    def __init__(self, cfg: EngineConfig, spec: EPSpec, device: str | torch.device = "cuda"):
        if spec.fused:
            spec.max_tokens = max(spec.max_tokens, cfg.max_batched_tokens + cfg.max_num_seqs)
        self.spec = spec
        self.engine = LLMEngine(cfg, device=device, ep=spec)
        self.idle_forwards = 0

    # request API: this rank's own requests
    def add_request(self, *a, **kw):
        return self.engine.add_request(*a, **kw)

    def abort_request(self, rid: str) -> None:
        self.engine.abort_request(rid)

    def has_unfinished(self) -> bool:
        return self.engine.has_unfinished()

    def _any_rank(self, mine: bool) -> bool:
        t = torch.tensor([1 if mine else 0], dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.spec.gloo)
        return bool(t.item())

    def step(self):
        """One lockstep iteration; every rank must call it the same number
        of times while any rank has work (``run_until_idle`` does)."""
        if not self._any_rank(self.engine.has_unfinished()):
            return []
        n0 = self.engine.runner.forwards
        outs = self.engine.step()
        if self.engine.runner.forwards == n0:
            self.engine.runner.idle_forward()
            self.idle_forwards += 1
        return outs

    def run_until_idle(self) -> dict[str, list[int]]:
        """Step until no rank has work; returns this rank's outputs."""
        got: dict[str, list[int]] = {}
        while self._any_rank(self.engine.has_unfinished()):
            n0 = self.engine.runner.forwards
            for o in self.engine.step():
                got.setdefault(o.request_id, []).extend(o.new_token_ids)
            if self.engine.runner.forwards == n0:
                self.engine.runner.idle_forward()
                self.idle_forwards += 1
        return got


class DPServed:
    """A data-parallel-attention rank as the engine-core server sees it: the
    server calls ``step`` every loop pass (``has_unfinished`` is always
    true), and every call is one lockstep vote of all ranks, so ranks with
    and without work stay in step. Everything else is this rank's engine."""

    def __init__(self, dp: DPAttentionEngine, idle_sleep_s: float = 0.0005):
        self.dp = dp
        self.engine = dp.engine
        self.idle_sleep_s = idle_sleep_s

    def __getattr__(self, name):
        return getattr(self.engine, name)

    def has_unfinished(self) -> bool:
        return True

    def step(self):
        import time

        if not self.dp._any_rank(self.engine.has_unfinished()):
            time.sleep(self.idle_sleep_s)
            return []
        n0 = self.engine.runner.forwards
        outs = self.engine.step()
        if self.engine.runner.forwards == n0:
            self.engine.runner.idle_forward()
            self.dp.idle_forwards += 1
        return outs

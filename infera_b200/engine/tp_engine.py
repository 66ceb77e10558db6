"""Tensor-parallel serving: replicated control, sharded compute.

Every rank of a tensor-parallel group runs the same scheduler, block
manager and sampler over its shard of the model (``DenseModel(tp=...)``).
Only rank 0 (the leader) talks to clients; before each engine step it
broadcasts the commands it applied since the previous step (request adds
and aborts, in order) over the group's gloo channel, and the followers
apply the same commands and step too. Deterministic scheduling plus
identical sampled tokens (the logits are all-gathered; per-request seeds
are process-independent) keep the replicas in lock step, so the only
per-token traffic is the model's own collectives on NVLink.

The leader is a drop-in for the engine in the engine core loop and the
offline ``generate``. Reference counterpart: the engines' tensor-parallel
workers (vLLM / SGLang launch one worker per GPU under a driver).
"""

from __future__ import annotations

import time

import torch.distributed as dist

from infera_b200.engine.request import SamplingParams

STOP = "stop"
HEARTBEAT_S = 0.5


class TPLeader:
    """Wraps rank 0's LLMEngine; everything but ``step`` is delegated."""

    def __init__(self, engine, group):
        self.engine = engine
        self.group = group
        engine.cmd_log = []
        self._last = time.monotonic()

    def __getattr__(self, name):
        return getattr(self.engine, name)

    def _broadcast(self, payload) -> None:
        obj = [payload]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        self._last = time.monotonic()

    def step(self):
        cmds, self.engine.cmd_log = self.engine.cmd_log, []
        cmds += self.engine.pd_tp_decisions()   # applied on this rank already
        self._broadcast(("step", cmds))
        return self.engine.step()

    def idle(self) -> None:
        """Keep followers' blocking receive alive while nothing runs."""
        if time.monotonic() - self._last >= HEARTBEAT_S:
            cmds, self.engine.cmd_log = self.engine.cmd_log, []
            self._broadcast(("idle", cmds))

    def shutdown(self) -> None:
        self._broadcast(STOP)

    def generate(self, prompts: list[list[int]], sampling: SamplingParams | None = None) -> list[list[int]]:
        ids = []
        for i, p in enumerate(prompts):
            rid = f"gen-{self.engine.num_steps}-{i}"
            self.engine.add_request(rid, p, sampling)
            ids.append(rid)
        outs: dict[str, list[int]] = {rid: [] for rid in ids}
        while self.engine.has_unfinished():
            for o in self.step():
                if o.request_id in outs:
                    outs[o.request_id].extend(o.new_token_ids)
        return [outs[r] for r in ids]


def follower_step(engine, group) -> bool:
    """Receive and mirror one leader message (commands, then the step);
    False once the leader said stop."""
    obj = [None]
    dist.broadcast_object_list(obj, src=0, group=group)
    msg = obj[0]
    if msg == STOP:
        return False
    kind, cmds = msg
    for c in cmds:
        if c[0] == "add":
            engine.add_request(c[1], c[2], c[3])
        elif c[0] == "abort":
            engine.abort_request(c[1])
        elif c[0].startswith("pd_"):
            engine.pd_apply(c)
    if kind == "step":  # mirror the leader's step exactly
        engine.step()
        engine.tp_steps = getattr(engine, "tp_steps", 0) + 1
    return True


def follower_loop(engine, group) -> int:
    """Run on ranks > 0 until the leader says stop; returns the step count."""
    n0 = getattr(engine, "tp_steps", 0)
    while follower_step(engine, group):
        pass
    return engine.tp_steps - n0 if hasattr(engine, "tp_steps") else 0

"""Policy construction from the server's flags."""

from __future__ import annotations

from infera_b200.router.policy.kv_aware import KvAwarePolicy
from infera_b200.router.policy.round_robin import RoundRobinPolicy

POLICY_NAMES = ("kv-aware", "round-robin")


def build_policy(name: str, *, tokenizer=None, overlap_weight: float = 1.0, prefill_overlap_weight=None,
                 decode_overlap_weight=None, kv_client=None, metrics=None, use_zmq: bool = True):
    if name == "round-robin":
        return RoundRobinPolicy()
    if name == "kv-aware":
        from infera_b200.router.kv_event.block_hasher import BlockHasher
        from infera_b200.router.kv_event.client import KvEventClient

        client = kv_client or KvEventClient(use_zmq=use_zmq)
        return KvAwarePolicy(client, BlockHasher(tokenizer), overlap_weight=overlap_weight,
                             prefill_overlap_weight=prefill_overlap_weight,
                             decode_overlap_weight=decode_overlap_weight, metrics=metrics)
    raise ValueError(f"unknown policy {name!r}; choose from {POLICY_NAMES}")

"""Round-robin over targets, with an independent rotation per candidate
set (so prefill and decode pools rotate separately)."""

from __future__ import annotations

from infera_b200.router.policy.base import Policy
from infera_b200.router.policy.target import expand_targets


class RoundRobinPolicy(Policy):
    name = "round-robin"

    def __init__(self) -> None:
        self._ctr: dict[tuple, int] = {}

    def pick(self, candidates, request, *, role_hint=None):
        targets = expand_targets(candidates)
        if not targets:
            raise LookupError("no candidates")
        key = (role_hint, tuple(sorted(t.route_key for t in targets)))
        i = self._ctr.get(key, 0)
        self._ctr[key] = i + 1
        return targets[i % len(targets)], []

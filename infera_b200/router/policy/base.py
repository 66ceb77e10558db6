"""Routing policy interface (``infera/router/policy/base.py:18-67``)."""

from __future__ import annotations

from abc import ABC, abstractmethod

from infera_b200.common.worker_pool import WorkerInfo
from infera_b200.router.policy.target import RouteTarget


class Policy(ABC):
    name = "base"

    @abstractmethod
    def pick(self, candidates: list[WorkerInfo], request: dict, *,
             role_hint: str | None = None) -> tuple[RouteTarget, list[int]]:
        """Choose a target; also return the request's block hashes (may be
        empty) so the router can report them as in flight."""

    def on_worker_added(self, worker: WorkerInfo) -> None:
        return None

    def on_worker_removed(self, worker_id: str) -> None:
        return None

    def on_request_started(self, route_key: str, blocks: list[int] | None = None) -> None:
        return None

    def on_request_finished(self, route_key: str, blocks: list[int] | None = None) -> None:
        return None

    @property
    def kv_client(self):
        return None

    async def aclose(self) -> None:
        return None

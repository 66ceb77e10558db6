"""Route targets: a worker, or one DP rank of a rank-multiplexed worker.

A worker registered with ``dp_size > 1`` and no fixed ``dp_rank`` expands
into one target per rank; its route key is ``<worker_id>#dp<rank>``
(``infera/router/policy/target.py:26-54``).
"""

from __future__ import annotations

from dataclasses import dataclass

from infera_b200.common.worker_pool import WorkerInfo


@dataclass(frozen=True)
class RouteTarget:
    worker: WorkerInfo
    dp_rank: int | None = None

    @property
    def route_key(self) -> str:
        if self.dp_rank is None or (self.worker.dp_size or 1) <= 1 or self.worker.dp_rank is not None:
            return self.worker.worker_id
        return f"{self.worker.worker_id}#dp{self.dp_rank}"


def expand_targets(workers: list[WorkerInfo]) -> list[RouteTarget]:
    out = []
    for w in workers:
        if w.dp_size and w.dp_size > 1 and w.dp_rank is None:
            out.extend(RouteTarget(w, r) for r in range(w.dp_size))
        else:
            out.append(RouteTarget(w, w.dp_rank))
    return out

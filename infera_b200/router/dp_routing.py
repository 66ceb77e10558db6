"""Data-parallel rank addressing.

A target bound to one DP rank of a rank-multiplexed worker carries the
``X-Data-Parallel-Rank`` header; PD room ids are aligned so that
``room % dp_size == prefill rank`` (``infera/router/dp_routing.py:22-57``).
"""

from __future__ import annotations

DP_RANK_HEADER = "X-Data-Parallel-Rank"


def dp_rank_header(target) -> dict:
    w = target.worker
    if target.dp_rank is not None and (w.dp_size or 1) > 1:
        return {DP_RANK_HEADER: str(target.dp_rank)}
    return {}


def align_room_to_prefill_rank(room: int, target) -> int:
    w = target.worker
    size = w.dp_size or 1
    if size <= 1 or target.dp_rank is None:
        return room
    return room - (room % size) + target.dp_rank


def disagg_prefill_dp_rank(target) -> int | None:
    return target.dp_rank if (target.worker.dp_size or 1) > 1 else None

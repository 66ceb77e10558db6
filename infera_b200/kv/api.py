"""HTTP surface of the tier-aware KV index (mounted by the router or run
alone): ``POST /v1/kv-index/match`` with ``{"model", "compat",
"token_ids", "block_size"}`` (or precomputed ``"blocks"``) returns every
publisher's per-tier overlap; ``GET /v1/kv-index/stats``. Publishers serve
``GET /v1/kv-index/snapshot`` from their probe. Role of ``infera/kv/api.py:50-209``.
"""

from __future__ import annotations

from fastapi import APIRouter
from fastapi.responses import JSONResponse

from infera_b200.kv.hashing import hash_prompt
from infera_b200.kv.types import BlockKey
from infera_b200.kv.wire import snapshot_json


def index_router(index) -> APIRouter:
    r = APIRouter()

    @r.post("/v1/kv-index/match")
    async def match(body: dict):
        model, compat = body.get("model"), body.get("compat")
        if not model or not compat:
            return JSONResponse({"error": "model and compat are required"}, status_code=400)
        if "blocks" in body:
            q = [BlockKey(int(a), int(b)) for a, b in body["blocks"]]
        else:
            q = hash_prompt(body.get("token_ids") or [], int(body.get("block_size") or 64), body.get("lora"))
        res = index.find_matches(model, compat, q)
        return {"query_blocks": len(q),
                "matches": {p: {t.value: n for t, n in ob.by_tier.items()} for p, ob in res.items()}}

    @r.get("/v1/kv-index/stats")
    async def stats():
        s = index.size()
        return {"trees": s.trees, "nodes": s.nodes, "optimistic": s.optimistic, "stored_events": s.stored_events,
                "removed_events": s.removed_events, "dropped_unknown_parent": s.dropped_unknown_parent}

    return r


def stats_router(plane) -> APIRouter:
    """``GET /v1/kv-stats``: counters of the router's index data plane
    (index, writer, subscribers, reconciler), as ``infera/kv/api.py:78-133``
    serves them."""
    r = APIRouter()

    @r.get("/v1/kv-stats")
    async def kv_stats():
        return plane.stats()

    return r


def publisher_router(probe) -> APIRouter:
    r = APIRouter()

    @r.get("/v1/kv-index/snapshot")
    async def snapshot():
        return snapshot_json(probe.publisher, probe.model, probe.compat, probe.chains())

    return r

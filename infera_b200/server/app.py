"""The HTTP front door.

Routes (paths and status codes of ``infera/server/app.py:110-619``):

    POST /v1/chat/completions, /v1/completions   OpenAI, streamed or not
    POST /v1/messages                            Anthropic Messages
    GET  /v1/models, /v1/workers
    GET  /v1/admin/cache-view/{worker_id}?dp_rank=
    POST /v1/admin/profile/{start|stop}          403 unless profiling is on
    GET|POST /v1/admin/scale                     404 unless the scaling API is on
    POST /v1/cache/prewarm                       202 / 400 / 503
    GET  /health, /metrics
    GET  /v1/kv-stats, /v1/kv-index/stats        tier-aware KV index counters
    POST /v1/kv-index/match                      per-publisher, per-tier prefix overlap

Every inference request is stamped with an ``X-Infera-Request-Id`` (body
field ``_infera_request_id`` while inside the router; response header on
the way out) and its cache hints; gateway headers ``x-worker-instance-id`` /
``x-prefill-instance-id`` select workers in direct mode.
"""

from __future__ import annotations

import json
import logging
import uuid
from dataclasses import dataclass, field

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse

from infera_b200.api.anthropic import (TranslationError, anthropic_to_openai_request, openai_to_anthropic_response,
                                       openai_to_anthropic_sse)
from infera_b200.router.cache_control import parse_cache_hints

logger = logging.getLogger(__name__)

REQUEST_ID_HEADER = "X-Infera-Request-Id"
WORKER_HEADER = "x-worker-instance-id"
PREFILL_HEADER = "x-prefill-instance-id"


@dataclass
class AppState:
    router: object
    registry: object
    policy: object = None
    metrics: object = None
    profiler: object = None          # ProfileFanout or None (disabled)
    scaler: object = None            # DeploymentScaler or None (disabled)
    kvd_client: object = None        # prefetch-hint sink or None
    block_size: int = 16
    kv_plane: object = None          # tier-aware KV index plane (infera_b200.kv.plane) or None
    extra: dict = field(default_factory=dict)


def _stash_gateway_headers(body: dict, request: Request) -> None:
    w = request.headers.get(WORKER_HEADER)
    p = request.headers.get(PREFILL_HEADER)
    if w:
        body["_infera_direct_worker"] = w
    if p:
        body["_infera_direct_prefill"] = p


def build_app(state: AppState) -> FastAPI:
    app = FastAPI(title="infera-b200")
    app.state.s = state
    if state.kv_plane is not None:
        from infera_b200.kv.api import index_router, stats_router

        app.include_router(stats_router(state.kv_plane))
        app.include_router(index_router(state.kv_plane.index))

    async def dispatch_inference(request: Request, path: str) -> Response:
        try:
            body = await request.json()
        except (ValueError, json.JSONDecodeError):
            return JSONResponse({"error": "invalid JSON body"}, status_code=400)
        if not isinstance(body, dict):
            return JSONResponse({"error": "body must be a JSON object"}, status_code=400)
        rid = request.headers.get(REQUEST_ID_HEADER) or uuid.uuid4().hex
        body["_infera_request_id"] = rid
        body["_infera_cache_hints"] = parse_cache_hints(body)
        if state.metrics is not None:
            state.metrics.cache_control_seen.labels(retention=body["_infera_cache_hints"].retention.value).inc()
        _stash_gateway_headers(body, request)
        stream = bool(body.get("stream", False))
        if state.metrics is not None:
            with state.metrics.track_request("front") as obs:
                resp = await state.router.dispatch(body, stream=stream, path=path)
                obs["outcome"] = str(resp.status_code) if resp.status_code >= 400 else "ok"
        else:
            resp = await state.router.dispatch(body, stream=stream, path=path)
        resp.headers[REQUEST_ID_HEADER] = rid
        return resp

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        return await dispatch_inference(request, "/v1/chat/completions")

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await dispatch_inference(request, "/v1/completions")

    @app.post("/v1/messages")
    async def messages(request: Request):
        try:
            body = await request.json()
        except (ValueError, json.JSONDecodeError):
            return JSONResponse({"type": "error", "error": {"type": "invalid_request_error",
                                                            "message": "invalid JSON"}}, status_code=400)
        ver = request.headers.get("anthropic-version")
        if ver:
            logger.debug("anthropic-version %s", ver)
        hints = parse_cache_hints(body)
        try:
            oa = anthropic_to_openai_request(body)
        except TranslationError as e:
            return JSONResponse({"type": "error", "error": {"type": "invalid_request_error", "message": str(e)}},
                                status_code=400)
        rid = request.headers.get(REQUEST_ID_HEADER) or uuid.uuid4().hex
        oa["_infera_request_id"] = rid
        oa["_infera_cache_hints"] = hints
        _stash_gateway_headers(oa, request)
        stream = oa["stream"]
        resp = await state.router.dispatch(oa, stream=stream, path="/v1/chat/completions")
        if resp.status_code >= 400:
            resp.headers[REQUEST_ID_HEADER] = rid
            return resp
        model = body.get("model")
        if stream and isinstance(resp, StreamingResponse):
            out = StreamingResponse(openai_to_anthropic_sse(resp.body_iterator, model),
                                    media_type="text/event-stream")
        else:
            try:
                obj = json.loads(resp.body)
            except (ValueError, AttributeError):
                return JSONResponse({"type": "error", "error": {"type": "api_error",
                                                                "message": "bad upstream response"}}, status_code=502)
            out = JSONResponse(openai_to_anthropic_response(obj, model))
        out.headers[REQUEST_ID_HEADER] = rid
        return out

    @app.get("/v1/models")
    async def models():
        pool = state.registry.pool
        data = [{"id": m, "object": "model", "owned_by": "infera-b200"} for m in pool.models()]
        return {"object": "list", "data": data}

    @app.get("/v1/workers")
    async def workers():
        return {"workers": [w.to_public() for w in state.registry.pool.all()]}

    @app.get("/v1/admin/cache-view/{worker_id}")
    async def cache_view(worker_id: str, dp_rank: int | None = None):
        client = getattr(state.policy, "kv_client", None)
        if client is None:
            return JSONResponse({"error": "policy has no KV view"}, status_code=404)
        if state.registry.pool.get(worker_id) is None:
            return JSONResponse({"error": f"unknown worker {worker_id!r}"}, status_code=404)
        view = client.cache_view(worker_id, dp_rank)
        out = {"worker_id": worker_id, "dp_rank": dp_rank, "num_blocks": len(view),
               "block_hashes": [str(h) for h in list(view)[:10000]]}
        if state.kv_plane is not None:   # blocks per tier (device / host / disk) in the tier-aware index
            out["index_tiers"] = state.kv_plane.index.tier_counts(worker_id)
        return out

    @app.post("/v1/admin/profile/{action}")
    async def profile(action: str, request: Request):
        if state.profiler is None:
            return JSONResponse({"error": "profiling is disabled (--enable-profiling)"}, status_code=403)
        if action not in ("start", "stop"):
            return JSONResponse({"error": f"unknown action {action!r}"}, status_code=404)
        try:
            body = await request.json()
        except Exception:
            body = {}
        res = await state.profiler.fan_out(action, body or {})
        code = 200 if res.get("targets") else 404
        return JSONResponse(res, status_code=code)

    @app.get("/v1/admin/scale")
    async def scale_get():
        if state.scaler is None:
            return JSONResponse({"error": "scaling API disabled (--enable-scaling-api)"}, status_code=404)
        try:
            return await state.scaler.get()
        except Exception as e:
            return JSONResponse({"error": str(e)}, status_code=502)

    @app.post("/v1/admin/scale")
    async def scale_post(request: Request):
        if state.scaler is None:
            return JSONResponse({"error": "scaling API disabled (--enable-scaling-api)"}, status_code=404)
        try:
            body = await request.json()
        except Exception:
            return JSONResponse({"error": "invalid JSON"}, status_code=400)
        from infera_b200.server.scaling import ScaleError

        try:
            return await state.scaler.scale(body)
        except ScaleError as e:
            return JSONResponse({"error": str(e)}, status_code=e.status)

    @app.post("/v1/cache/prewarm")
    async def prewarm(request: Request):
        try:
            body = await request.json()
        except Exception:
            return JSONResponse({"error": "invalid JSON"}, status_code=400)
        if not isinstance(body, dict) or not (body.get("prompt") or body.get("messages")):
            return JSONResponse({"error": "prewarm needs a prompt or messages"}, status_code=400)
        if state.kvd_client is None:
            return JSONResponse({"error": "no KV tier daemon configured"}, status_code=503)
        from infera_b200.router.kv_event.block_hasher import BlockHasher

        hasher = getattr(state.policy, "_hasher", None) or BlockHasher()
        hashes = hasher.hash_for(body, block_size=state.block_size)
        ok = await state.kvd_client.prefetch_hint(hashes, retention=parse_cache_hints(body).retention.value)
        if not ok:
            return JSONResponse({"error": "KV tier daemon unreachable"}, status_code=503)
        return JSONResponse({"accepted": True, "blocks": len(hashes)}, status_code=202)

    @app.get("/health")
    async def health():
        return {"status": "ok", "workers": len(state.registry.pool.list_active())}

    @app.get("/metrics")
    async def metrics():
        if state.metrics is None:
            return Response(b"", media_type="text/plain")
        state.metrics.snapshot_pool(state.registry.pool, getattr(state.policy, "kv_client", None))
        return Response(state.metrics.render(), media_type="text/plain; version=0.0.4")

    return app

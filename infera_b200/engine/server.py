"""The worker's OpenAI-compatible HTTP server (one engine instance).

Routes: POST /v1/completions, /v1/chat/completions (streamed SSE or JSON),
GET /v1/models, /health, /metrics, /v1/kv-snapshot, POST /start_profile,
/stop_profile.

Request fields beyond OpenAI's: ``prompt`` may be a list of token ids;
``ignore_eos``, ``stop_token_ids``, ``min_tokens``, ``seed``;
``return_token_ids`` puts ``token_ids`` on every choice (and
``prompt_token_ids`` on the first chunk) for router-side migration;
``kv_transfer_params.infera_retention`` carries the retention hint.

While draining, new requests get 503 and handed-back streams end with an
error event carrying the draining notice (the router migrates them).
"""

from __future__ import annotations

import json
import time
import uuid

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse

from infera_b200.engine.async_engine import HANDBACK
from infera_b200.engine.request import SamplingParams
from infera_b200.router.transport import DRAINING_NOTICE
from infera_b200.utils.tokenizer import request_token_ids


def _sampling(body: dict, default_max: int) -> SamplingParams:
    mt = body.get("max_tokens") or body.get("max_completion_tokens") or default_max
    stop_ids = body.get("stop_token_ids") or []
    ktp = body.get("kv_transfer_params") or {}
    return SamplingParams(max_tokens=int(mt), temperature=float(body.get("temperature") or 0.0),
                          seed=body.get("seed"), stop_token_ids=[int(x) for x in stop_ids],
                          ignore_eos=bool(body.get("ignore_eos", False)), min_tokens=int(body.get("min_tokens", 0)),
                          retention=ktp.get("infera_retention") or body.get("infera_retention"),
                          kv_transfer={k: v for k, v in ktp.items() if k != "infera_retention"} or None)


def _sse(obj: dict) -> bytes:
    return b"data: " + json.dumps(obj, separators=(",", ":")).encode() + b"\n\n"


def build_worker_app(aeng, tokenizer, model_name: str, extra_metrics=None) -> FastAPI:
    app = FastAPI(title="infera-b200 worker")
    app.state.aeng = aeng

    async def run(body: dict, chat: bool):
        if aeng.draining:
            return JSONResponse({"error": {"message": DRAINING_NOTICE, "type": "unavailable"}}, status_code=503)
        try:
            ids = request_token_ids(body, tokenizer)
        except Exception as e:
            return JSONResponse({"error": {"message": f"bad prompt: {e}", "type": "invalid_request"}},
                                status_code=400)
        if not ids:
            return JSONResponse({"error": {"message": "empty prompt", "type": "invalid_request"}}, status_code=400)
        sp = _sampling(body, 256)
        rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex
        want_ids = bool(body.get("return_token_ids"))
        stream = bool(body.get("stream"))
        include_usage = bool((body.get("stream_options") or {}).get("include_usage"))
        created = int(time.time())
        obj_kind = "chat.completion.chunk" if chat else "text_completion"

        def choice(new_ids, finish):
            text = tokenizer.decode(new_ids) if new_ids else ""
            if chat:
                c = {"index": 0, "delta": {"content": text} if text or finish is None else {}, "finish_reason": finish}
            else:
                c = {"index": 0, "text": text, "finish_reason": finish}
            if want_ids:
                c["token_ids"] = list(new_ids)
            return c

        if stream:
            async def gen():
                first = True
                n_out = 0
                try:
                    async for o in aeng.generate(rid, ids, sp):
                        if o is HANDBACK:
                            yield _sse({"error": DRAINING_NOTICE})
                            return
                        if o.finish_reason and o.finish_reason.startswith("error"):
                            yield _sse({"error": o.finish_reason})
                            return
                        n_out += len(o.new_token_ids)
                        chunk = {"id": rid, "object": obj_kind, "created": created, "model": model_name,
                                 "choices": [choice(o.new_token_ids, o.finish_reason if o.finished else None)]}
                        if first and want_ids:
                            chunk["prompt_token_ids"] = ids
                        first = False
                        yield _sse(chunk)
                        if o.finished and include_usage:
                            yield _sse({"id": rid, "object": obj_kind, "created": created, "model": model_name,
                                        "choices": [], "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out,
                                                                 "total_tokens": len(ids) + n_out,
                                                                 "prompt_tokens_details": {
                                                                     "cached_tokens": o.num_cached_tokens}}})
                    yield b"data: [DONE]\n\n"
                except RuntimeError as e:
                    yield _sse({"error": str(e)})

            return StreamingResponse(gen(), media_type="text/event-stream")

        out_ids: list[int] = []
        finish = None
        cached = 0
        try:
            async for o in aeng.generate(rid, ids, sp):
                if o is HANDBACK:
                    return JSONResponse({"error": {"message": DRAINING_NOTICE}}, status_code=503)
                if o.finish_reason and o.finish_reason.startswith("error"):
                    return JSONResponse({"error": {"message": o.finish_reason}}, status_code=500)
                out_ids.extend(o.new_token_ids)
                if o.finished:
                    finish = o.finish_reason
                    cached = o.num_cached_tokens
        except RuntimeError as e:
            return JSONResponse({"error": {"message": str(e)}}, status_code=503)
        text = tokenizer.decode(out_ids)
        if chat:
            ch = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": finish}
        else:
            ch = {"index": 0, "text": text, "finish_reason": finish}
        if want_ids:
            ch["token_ids"] = out_ids
        resp = {"id": rid, "object": "chat.completion" if chat else "text_completion", "created": created,
                "model": model_name, "choices": [ch],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out_ids),
                          "total_tokens": len(ids) + len(out_ids),
                          "prompt_tokens_details": {"cached_tokens": cached}}}
        if want_ids:
            resp["prompt_token_ids"] = ids
        return JSONResponse(resp)

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await run(await request.json(), chat=False)

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await run(await request.json(), chat=True)

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "infera-b200"}]}

    @app.get("/health")
    async def health():
        if aeng.errors and aeng.last_error and "CUDA" in aeng.last_error:
            return JSONResponse({"status": "unhealthy", "error": aeng.last_error}, status_code=500)
        return {"status": "draining" if aeng.draining else "ok"}

    @app.get("/metrics")
    async def metrics():
        s = await aeng.stats_async()
        lines = []

        def g(name, v, help_):
            lines.append(f"# HELP {name} {help_}\n# TYPE {name} gauge\n{name}{{model_name=\"{model_name}\"}} {v}")

        g("infera_engine:num_requests_running", s["running"], "Requests in the running batch")
        g("infera_engine:num_requests_waiting", s["waiting"], "Requests queued")
        g("infera_engine:num_requests_inflight", s["inflight"], "Admitted and unfinished requests")
        g("infera_engine:kv_cache_usage_perc", round(s["kv_usage"], 6), "Fraction of KV pages in use")
        g("infera_engine:prefix_cache_hit_rate", round(s["prefix_hit_rate"], 6), "Prompt tokens served from cache")
        g("infera_engine:pd_push_queue", s.get("pd_push_queue", 0), "KV pushes not yet acknowledged")
        g("infera_engine:pd_pushes_total", s.get("pd_pushes", 0), "KV pushes completed")
        g("infera_engine:pd_push_bytes_total", s.get("pd_push_bytes", 0), "KV bytes pushed to decode instances")
        g("infera_engine:pd_push_seconds_total", round(s.get("pd_push_seconds", 0.0), 6), "Launch-to-done push time")
        g("infera_engine:pd_push_device_seconds_total", round(s.get("pd_push_device_seconds", 0.0), 6),
          "Device time of the push kernels")
        g("infera_engine:pd_parked", s.get("pd_parked", 0), "Requests waiting for pushed KV")
        g("infera_engine:generation_tokens_total", s["generation_tokens"], "Generated tokens")
        g("infera_engine:prompt_tokens_total", s["prompt_tokens"], "Computed prompt tokens")
        g("infera_engine:steps_total", s.get("steps", 0), "Engine steps that ran a forward")
        g("infera_engine:forward_seconds_total", round(s.get("forward_s", 0.0), 6),
          "Host time inside model forwards (each ends on its sampled tokens)")
        # names the reference's drain reader understands
        g("vllm:num_requests_running", s["running"], "alias")
        g("vllm:num_requests_waiting", s["waiting"], "alias")
        if extra_metrics is not None:
            lines.extend(extra_metrics())
        return Response("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    @app.get("/v1/kv-snapshot")
    async def kv_snapshot(model: str | None = None, compat_key: str | None = None):
        """Without parameters: the device prefix cache's block hashes (the
        router's seed-0 chain). With ``model`` and ``compat_key``: this
        instance's chains in the tier-aware KV index (device / host / disk),
        what the router's reconciler pulls."""
        if model is None and compat_key is None:
            return await aeng.kv_snapshot()
        snap = await aeng.kv_index_snapshot()
        if "error" in snap:
            return JSONResponse(snap, status_code=404)
        if (model is not None and snap.get("model") != model) or (
                compat_key is not None and snap.get("compat") != compat_key):
            return JSONResponse({"error": "no snapshot for that model / compat key"}, status_code=404)
        return snap

    @app.post("/start_profile")
    async def start_profile(request: Request):
        res = await aeng.start_profile()
        return JSONResponse(res, status_code=409 if "error" in res else 200)

    @app.post("/stop_profile")
    async def stop_profile(request: Request):
        res = await aeng.stop_profile()
        return JSONResponse(res, status_code=409 if res.get("error") == "not profiling" else 200)

    return app

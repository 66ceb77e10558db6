"""Front door, Anthropic translation, etcd discovery/registration, and the
routers (failover, migration, PD dual dispatch) against mock workers."""

import asyncio
import json

import httpx
import pytest
from fastapi.testclient import TestClient

from infera_b200.api.anthropic import (TranslationError, anthropic_to_openai_request, openai_to_anthropic_response,
                                       openai_to_anthropic_sse)
from infera_b200.common.discovery import EtcdRegistry, InProcessRegistry
from infera_b200.common.etcd_fake import build_app as etcd_app
from infera_b200.common.registration import EtcdRegistration
from infera_b200.common.worker_pool import DisaggMode, WorkerInfo
from infera_b200.router.auto import AutoRouter
from infera_b200.router.breaker import CircuitBreaker
from infera_b200.router.mixed import MixedRouter
from infera_b200.router.policy.round_robin import RoundRobinPolicy
from infera_b200.router.transport import HttpTransport
from infera_b200.server.app import AppState, build_app
from infera_b200.server.metrics import RouterMetrics


# ---------------------------------------------------------------- Anthropic
def test_anthropic_request_translation():
    body = {"model": "m", "max_tokens": 64, "system": [{"type": "text", "text": "sys"}],
            "stop_sequences": ["END"], "temperature": 0.2,
            "tools": [{"name": "get", "description": "d", "input_schema": {"type": "object"}}],
            "tool_choice": {"type": "any"},
            "messages": [
                {"role": "user", "content": "hello"},
                {"role": "assistant", "content": [{"type": "text", "text": "calling"},
                                                  {"type": "tool_use", "id": "t1", "name": "get",
                                                   "input": {"a": 1}}]},
                {"role": "user", "content": [{"type": "tool_result", "tool_use_id": "t1", "content": "42"}]}]}
    oa = anthropic_to_openai_request(body)
    assert oa["messages"][0] == {"role": "system", "content": "sys"}
    assert oa["messages"][2]["tool_calls"][0]["function"]["arguments"] == json.dumps({"a": 1})
    assert oa["messages"][3] == {"role": "tool", "tool_call_id": "t1", "content": "42"}
    assert oa["tool_choice"] == "required" and oa["stop"] == ["END"]
    assert oa["tools"][0]["function"]["parameters"] == {"type": "object"}


def test_anthropic_rejects_media_and_missing_max_tokens():
    with pytest.raises(TranslationError):
        anthropic_to_openai_request({"max_tokens": 5, "messages": [{"role": "user", "content": [
            {"type": "image", "source": {"type": "base64", "data": "xx"}}]}]})
    with pytest.raises(TranslationError):
        anthropic_to_openai_request({"messages": []})


def test_anthropic_response_and_sse():
    resp = {"model": "m", "choices": [{"message": {"content": "hi", "tool_calls": [
        {"id": "c1", "function": {"name": "f", "arguments": "{\"x\": 2}"}}]}, "finish_reason": "tool_calls"}],
        "usage": {"prompt_tokens": 3, "completion_tokens": 4}}
    a = openai_to_anthropic_response(resp)
    assert a["stop_reason"] == "tool_use" and a["content"][1]["input"] == {"x": 2}
    assert a["usage"] == {"input_tokens": 3, "output_tokens": 4}

    async def chunks():
        for t in ("He", "llo"):
            yield b'data: {"choices":[{"delta":{"content":"' + t.encode() + b'"}}]}\n\n'
        yield b'data: {"choices":[{"delta":{},"finish_reason":"length"}],"usage":{"prompt_tokens":2,"completion_tokens":2}}\n\n'
        yield b"data: [DONE]\n\n"

    async def collect():
        return [x async for x in openai_to_anthropic_sse(chunks(), "m")]

    evs = asyncio.run(collect())
    kinds = [e.split(b"\n")[0] for e in evs]
    assert kinds[0] == b"event: message_start" and kinds[-1] == b"event: message_stop"
    assert b"text_delta" in b"".join(evs) and b'"max_tokens"' in b"".join(evs)


# ---------------------------------------------------------------- mock workers via httpx.MockTransport
def _sse(tokens, ids=True):
    out = b""
    for i, t in enumerate(tokens):
        ch = {"index": 0, "text": "x", "finish_reason": "length" if i == len(tokens) - 1 else None}
        if ids:
            ch["token_ids"] = [t]
        out += b"data: " + json.dumps({"choices": [ch]}).encode() + b"\n\n"
    return out + b"data: [DONE]\n\n"


def _router(pool, handler, cls=MixedRouter, migration_limit=0, retries=1):
    client = httpx.AsyncClient(transport=httpx.MockTransport(handler))
    return cls(pool, RoundRobinPolicy(), transport=HttpTransport(client), breaker=CircuitBreaker(),
               request_max_retries=retries, migration_limit=migration_limit)


def _pool(n=2, mode=DisaggMode.MIXED, meta=None):
    reg = InProcessRegistry()
    for i in range(n):
        reg.register(WorkerInfo(f"w{i}", f"http://w{i}", "m", disagg_mode=mode, disagg_meta=meta or {},
                                kv_block_size=16).to_payload())
    return reg


async def _read(resp):
    if hasattr(resp, "body_iterator"):
        return b"".join([c async for c in resp.body_iterator])
    return resp.body


def test_failover_before_first_byte():
    calls = []

    def handler(req):
        calls.append(req.url.host)
        if req.url.host == "w0":
            return httpx.Response(500, json={"error": "boom"})
        return httpx.Response(200, content=_sse([1, 2]))

    reg = _pool()
    r = _router(reg.pool, handler)

    async def go():
        out = []
        for _ in range(2):
            resp = await r.dispatch({"model": "m", "prompt": [1], "stream": True}, stream=True, path="/v1/completions")
            out.append((resp.status_code, await _read(resp)))
        return out

    res = asyncio.run(go())
    assert all(s == 200 and b"[DONE]" in b for s, b in res)
    assert "w0" in calls and calls.count("w1") == 2


def test_migration_after_midstream_break():
    def handler(req):
        body = json.loads(req.content)
        if req.url.host == "w0":
            # two tokens then the stream ends without [DONE]
            return httpx.Response(200, content=b"".join(
                b"data: " + json.dumps({"prompt_token_ids": [9, 9] if i == 0 else None,
                                        "choices": [{"index": 0, "text": "x", "token_ids": [t]}]}).encode() + b"\n\n"
                for i, t in enumerate([5, 6])))
        assert body["prompt"] == [9, 9, 5, 6] and body["max_tokens"] == 2
        return httpx.Response(200, content=_sse([7, 8]))

    reg = _pool()
    r = _router(reg.pool, handler, migration_limit=1)

    async def go():
        resp = await r.dispatch({"model": "m", "prompt": [9, 9], "max_tokens": 4, "stream": True}, stream=True,
                                path="/v1/completions")
        return await _read(resp)

    out = asyncio.run(go())
    assert out.count(b"data: ") >= 5 and out.rstrip().endswith(b"[DONE]")
    assert b"token_ids" not in out  # stripped before the client


def test_auto_router_pd_and_empty_pool():
    seen = []

    def handler(req):
        body = json.loads(req.content)
        seen.append((req.url.host, body.get("max_tokens"), body.get("kv_transfer_params")))
        if req.url.host == "p0":
            return httpx.Response(200, json={"choices": [{"text": "x"}]})
        return httpx.Response(200, content=_sse([1, 2, 3]))

    meta = {"protocol": "b200-nvlink-push", "params": {}}
    reg = InProcessRegistry()
    reg.register(WorkerInfo("p0", "http://p0", "m", disagg_mode=DisaggMode.PREFILL, disagg_meta=meta).to_payload())
    r = _router(reg.pool, handler, cls=AutoRouter)

    async def go(stream):
        resp = await r.dispatch({"model": "m", "prompt": [1, 2], "max_tokens": 4, "stream": stream}, stream=stream,
                                path="/v1/completions")
        return resp.status_code, await _read(resp)

    code, body = asyncio.run(go(True))
    assert code == 503 and b"decode" in body
    reg.register(WorkerInfo("d0", "http://d0", "m", disagg_mode=DisaggMode.DECODE, disagg_meta=meta).to_payload())
    code, body = asyncio.run(go(True))
    assert code == 200 and b"[DONE]" in body
    legs = {h: (mt, k) for h, mt, k in seen}
    assert legs["p0"][0] == 1 and legs["p0"][1]["do_remote_decode"]
    assert legs["d0"][0] == 4 and legs["d0"][1]["do_remote_prefill"]  # decode keeps the full budget
    assert legs["p0"][1]["room"] == legs["d0"][1]["room"]


# ---------------------------------------------------------------- app routes
class _FakeRouter:
    def __init__(self):
        self.bodies = []

    async def dispatch(self, body, *, stream, path):
        from fastapi.responses import JSONResponse, StreamingResponse

        self.bodies.append((path, body))
        if stream:
            async def gen():
                yield b'data: {"choices":[{"delta":{"content":"ok"}}]}\n\n'
                yield b"data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        return JSONResponse({"choices": [{"message": {"content": "ok"}, "finish_reason": "stop"}],
                             "usage": {"prompt_tokens": 1, "completion_tokens": 1}})


def test_app_routes():
    reg = _pool(2)
    fr = _FakeRouter()
    app = build_app(AppState(router=fr, registry=reg, metrics=RouterMetrics()))
    c = TestClient(app)
    r = c.post("/v1/chat/completions", json={"model": "m", "messages": [{"role": "user", "content": "x"}]},
               headers={"x-worker-instance-id": "w1"})
    assert r.status_code == 200 and r.headers["X-Infera-Request-Id"]
    path, body = fr.bodies[-1]
    assert body["_infera_direct_worker"] == "w1" and "_infera_cache_hints" in body
    assert c.post("/v1/completions", content=b"{bad").status_code == 400
    r = c.post("/v1/messages", json={"model": "m", "max_tokens": 4, "messages": [{"role": "user", "content": "x"}]})
    assert r.status_code == 200 and r.json()["type"] == "message"
    r = c.post("/v1/messages", json={"model": "m", "max_tokens": 4, "stream": True,
                                     "messages": [{"role": "user", "content": "x"}]})
    assert b"message_start" in r.content
    assert c.post("/v1/messages", json={"messages": []}).status_code == 400
    assert {m["id"] for m in c.get("/v1/models").json()["data"]} == {"m"}
    assert len(c.get("/v1/workers").json()["workers"]) == 2
    assert c.post("/v1/admin/profile/start", json={}).status_code == 403
    assert c.get("/v1/admin/scale").status_code == 404
    assert c.post("/v1/cache/prewarm", json={"prompt": [1, 2]}).status_code == 503
    assert c.post("/v1/cache/prewarm", json={}).status_code == 400
    assert c.get("/health").json()["workers"] == 2
    assert b"infera_active_workers" in c.get("/metrics").content


# ---------------------------------------------------------------- etcd discovery + registration
def test_etcd_registry_lease_lifecycle():
    from infera_b200.bench.fleet import ServerThread, free_port

    srv = ServerThread(etcd_app(), free_port()).start()
    url = f"http://127.0.0.1:{srv.port}"

    async def go():
        reg = EtcdRegistry(url, reconnect_s=0.1)
        added, removed = [], []
        reg.on_worker_added(lambda w: added.append(w.worker_id))
        reg.on_worker_removed(lambda w: removed.append(w.worker_id))
        await reg.start()
        a = EtcdRegistration(url, WorkerInfo("h:1", "http://h:1", "m").to_payload(), lease_ttl=30)
        await a.register()
        for _ in range(100):
            if reg.pool.get("h:1"):
                break
            await asyncio.sleep(0.02)
        assert added == ["h:1"]
        # the lease vanishes (as if it expired): keepalive re-registers
        srv.server.config.app.state.etcd.revoke(a.lease_id)
        for _ in range(100):
            if removed:
                break
            await asyncio.sleep(0.02)
        assert removed == ["h:1"]
        assert await a.keepalive_once() is False and a.reregistrations == 1
        for _ in range(100):
            if reg.pool.get("h:1"):
                break
            await asyncio.sleep(0.02)
        assert reg.pool.get("h:1") is not None
        await a.deregister()
        for _ in range(100):
            if reg.pool.get("h:1") is None:
                break
            await asyncio.sleep(0.02)
        assert reg.pool.get("h:1") is None
        await a.close()
        await reg.stop()

    try:
        asyncio.run(go())
    finally:
        srv.stop()


def test_canary_mismatch_rejected():
    from infera_b200.common.worker_pool import KvRegistrationMetadata

    reg = InProcessRegistry()

    def rec(wid, canary):
        kv = KvRegistrationMetadata(16, 16, "t", "d", canary)
        return WorkerInfo(wid, f"http://{wid}", "m", kv=kv).to_payload()

    assert reg.register(rec("a", [1, 2, 3]))
    assert not reg.register(rec("b", [1, 2, 4]))
    assert "b" in reg.rejected and reg.pool.get("b") is None


# ---------------------------------------------------------------- CPU fleet (config 1 shape, shortened)
def test_fleet_kv_routing_and_drain():
    from infera_b200.bench.fleet import run_fleet

    res = asyncio.run(run_fleet(workers=3, rate=12.0, duration=8.0, drain_at=4.0, sessions=12, decode_ms=2.0))
    assert res["errors"] == 0
    assert res["drain"]["drained"] and res["drain"]["router_removed"]
    assert res["prefix_hit_rate"] > 0.5
    assert sum(v > 0 for v in res["router_view_blocks"].values()) >= 2

"""GAIE endpoint picker: PD-preferred picks with policy bookkeeping, the
ext_proc protobuf codec, and the gRPC server end to end (in-process)."""

import asyncio
import json

from infera_b200.common.worker_pool import DisaggMode, WorkerInfo, WorkerPool
from infera_b200.gaie import extproc as X
from infera_b200.gaie.picker import DEST_HEADER, PREFILL_HEADER, WORKER_HEADER, EndpointPicker
from infera_b200.router.policy.factory import build_policy


def _pool(pd: bool):
    pool = WorkerPool()
    if pd:
        pool.add(WorkerInfo("p0", "http://10.0.0.1:9000", "m", disagg_mode=DisaggMode.PREFILL, kv_block_size=16))
        pool.add(WorkerInfo("d0", "http://10.0.0.2:9000", "m", disagg_mode=DisaggMode.DECODE, kv_block_size=16))
    else:
        pool.add(WorkerInfo("w0", "http://10.0.0.3:9000", "m", kv_block_size=16))
    return pool


def test_picker_pd_and_release():
    pol = build_policy("kv-aware", use_zmq=False)
    pk = EndpointPicker(_pool(True), pol, target_port=8000)
    r = pk.pick("m", {"model": "m", "prompt": list(range(64))})
    assert r.destination == "10.0.0.2:8000" and r.prefill_id == "p0"
    h = r.headers()
    assert h[WORKER_HEADER] == "d0" and h[PREFILL_HEADER] == "p0" and h[DEST_HEADER] == "10.0.0.2:8000"
    assert pol.active_blocks("d0") == 4
    pk.release(r)
    assert pol.active_blocks("d0") == 0 and pol.active_blocks("p0") == 0
    assert EndpointPicker(WorkerPool(), pol).pick("m", {}) is None


def test_codec_roundtrip():
    raw = X.encode_request("request_headers", headers={":path": "/v1/chat/completions", "x-a": "b"},
                           end_of_stream=False)
    kind, d = X.decode_request(raw)
    assert kind == "request_headers" and d["headers"]["x-a"] == "b" and not d["end_of_stream"]
    kind, d = X.decode_request(X.encode_request("request_body", body=b"{}", end_of_stream=True))
    assert kind == "request_body" and d["body"] == b"{}" and d["end_of_stream"]
    f, res = X.decode_response(X.response(3, X.common_response({"k": "v"}, b"abc", True, True)))
    assert f == 3 and res["headers"] == {"k": "v"} and res["body"] == b"abc" and res["clear_route_cache"]


def test_grpc_server_routes_on_body():
    import grpc

    async def go():
        pol = build_policy("kv-aware", use_zmq=False)
        pk = EndpointPicker(_pool(False), pol)
        srv, ep, port = await X.serve(pk, host="127.0.0.1", port=0)
        try:
            async with grpc.aio.insecure_channel(f"127.0.0.1:{port}") as ch:
                call = ch.stream_stream(f"/{X.SERVICE}/{X.METHOD}", request_serializer=lambda b: b,
                                        response_deserializer=lambda b: b)
                body = json.dumps({"model": "m", "prompt": list(range(40))}).encode()

                async def reqs():
                    yield X.encode_request("request_headers", headers={":path": "/v1/completions"})
                    yield X.encode_request("request_body", body=body[:10], end_of_stream=False)
                    yield X.encode_request("request_body", body=body[10:], end_of_stream=True)

                out = [X.decode_response(r) async for r in call(reqs())]
        finally:
            await srv.stop(None)
        return out, ep.stats, pol

    out, stats, pol = asyncio.run(go())
    assert [f for f, _ in out] == [1, 3]
    assert out[1][1]["headers"][WORKER_HEADER] == "w0" and out[1][1]["body"].startswith(b'{"model"')
    assert stats["picks"] == 1 and pol.active_blocks("w0") == 0  # released at stream end

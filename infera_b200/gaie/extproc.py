"""Envoy external-processing (ext_proc v3) server for the endpoint picker.

gRPC ``envoy.service.ext_proc.v3.ExternalProcessor/Process`` (bidirectional
stream; one stream = one HTTP request). The messages are encoded and
decoded here by a small protobuf wire codec (varint / length-delimited
fields) for the subset the picker uses, with the upstream field numbers:
no protoc or Envoy proto packages are needed, and grpcio's generic handler
carries the bytes.

Flow (full-duplex streamed body): request headers without end-of-stream ->
CONTINUE; request body chunks are collected until end-of-stream, then the
picker routes on the JSON body and the answer carries the routing headers
(header mutation, route cache cleared) and echoes the body back as the
streamed body response; response phases pass through. The picker's
bookkeeping is released when the stream ends. Role of
``infera/gaie/ext_proc_server.py:65-186``.
"""

from __future__ import annotations

import json
import logging

logger = logging.getLogger(__name__)

SERVICE = "envoy.service.ext_proc.v3.ExternalProcessor"
METHOD = "Process"
OVERWRITE_IF_EXISTS_OR_ADD = 2


# ---------------------------------------------------------------- wire codec
def _varint(n: int) -> bytes:
    out = bytearray()
    n &= (1 << 64) - 1
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wt: int) -> bytes:
    return _varint((field << 3) | wt)


def f_bytes(field: int, data: bytes) -> bytes:
    return _key(field, 2) + _varint(len(data)) + data


def f_varint(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v) if v else b""


def parse(buf: bytes) -> dict[int, list]:
    """field number -> list of values (ints for varints, bytes otherwise)."""
    out: dict[int, list] = {}
    i, n = 0, len(buf)

    def varint():
        nonlocal i
        shift = res = 0
        while True:
            b = buf[i]
            i += 1
            res |= (b & 0x7F) << shift
            if not b & 0x80:
                return res
            shift += 7

    while i < n:
        k = varint()
        f, wt = k >> 3, k & 7
        if wt == 0:
            v = varint()
        elif wt == 2:
            ln = varint()
            v = buf[i:i + ln]
            i += ln
        elif wt == 1:
            v = buf[i:i + 8]
            i += 8
        elif wt == 5:
            v = buf[i:i + 4]
            i += 4
        else:
            raise ValueError(f"unsupported wire type {wt}")
        out.setdefault(f, []).append(v)
    return out


# ProcessingRequest oneof: 2 request_headers, 3 response_headers, 4 request_body,
# 5 response_body, 6 request_trailers, 7 response_trailers
REQ_KINDS = {2: "request_headers", 3: "response_headers", 4: "request_body", 5: "response_body",
             6: "request_trailers", 7: "response_trailers"}


def decode_request(raw: bytes) -> tuple[str, dict]:
    top = parse(raw)
    for f, kind in REQ_KINDS.items():
        if f in top:
            inner = parse(top[f][0])
            if kind.endswith("_body"):          # HttpBody: body=1, end_of_stream=2
                return kind, {"body": bytes(inner.get(1, [b""])[0]), "end_of_stream": bool(inner.get(2, [0])[0])}
            if kind.endswith("_headers"):       # HttpHeaders: headers=1 (HeaderMap), end_of_stream=3
                hdrs = {}
                for hv in parse(inner[1][0]).get(1, []) if 1 in inner else []:
                    d = parse(hv)
                    k = bytes(d.get(1, [b""])[0]).decode()
                    v = bytes(d.get(3, d.get(2, [b""]))[0]).decode()
                    hdrs[k] = v
                return kind, {"headers": hdrs, "end_of_stream": bool(inner.get(3, [0])[0])}
            return kind, {}
    return "unknown", {}


def encode_request(kind: str, **kw) -> bytes:
    """Client side (tests, tools): build a ProcessingRequest."""
    f = {v: k for k, v in REQ_KINDS.items()}[kind]
    if kind.endswith("_body"):
        inner = f_bytes(1, kw.get("body", b"")) + f_varint(2, int(kw.get("end_of_stream", False)))
    elif kind.endswith("_headers"):
        hm = b"".join(f_bytes(1, f_bytes(1, k.encode()) + f_bytes(3, v.encode()))
                      for k, v in (kw.get("headers") or {}).items())
        inner = f_bytes(1, hm) + f_varint(3, int(kw.get("end_of_stream", False)))
    else:
        inner = b""
    return f_bytes(f, inner)


def _header_option(k: str, v: str) -> bytes:
    return f_bytes(1, f_bytes(1, k.encode()) + f_bytes(3, v.encode())) + f_varint(3, OVERWRITE_IF_EXISTS_OR_ADD)


def common_response(headers: dict | None = None, body: bytes | None = None, end_of_stream: bool = True,
                    clear_route_cache: bool = False) -> bytes:
    out = b""
    if headers:
        out += f_bytes(2, b"".join(f_bytes(1, _header_option(k, v)) for k, v in headers.items()))
    if body is not None:  # BodyMutation.streamed_response (3) {body=1, end_of_stream=2}
        out += f_bytes(3, f_bytes(3, f_bytes(1, body) + f_varint(2, int(end_of_stream))))
    if clear_route_cache:
        out += f_varint(5, 1)
    return out


# ProcessingResponse oneof: 1 request_headers, 2 response_headers, 3 request_body,
# 4 response_body, 5 request_trailers, 6 response_trailers
def response(field: int, common: bytes = b"") -> bytes:
    inner = f_bytes(1, common) if field <= 4 else b""
    return f_bytes(field, inner)


def decode_response(raw: bytes) -> tuple[int, dict]:
    top = parse(raw)
    f = next(iter(top))
    inner = parse(top[f][0]) if top[f][0] else {}
    res = {"headers": {}, "body": None, "clear_route_cache": False}
    if 1 in inner and f <= 4:
        common = parse(inner[1][0])
        for hvo in parse(common[2][0]).get(1, []) if 2 in common else []:
            hv = parse(parse(hvo)[1][0])
            res["headers"][bytes(hv[1][0]).decode()] = bytes(hv.get(3, hv.get(2, [b""]))[0]).decode()
        if 3 in common:
            sr = parse(parse(common[3][0])[3][0])
            res["body"] = bytes(sr.get(1, [b""])[0])
        res["clear_route_cache"] = bool(common.get(5, [0])[0])
    return f, res


# ---------------------------------------------------------------- server
class ExtProcServer:
    def __init__(self, picker):
        self.picker = picker
        self.stats = {"streams": 0, "picks": 0, "no_pick": 0}

    def _route(self, raw: bytes):
        body = {}
        if raw:
            try:
                d = json.loads(raw)
                body = d if isinstance(d, dict) else {}
            except ValueError:
                pass
        try:
            r = self.picker.pick(body.get("model"), body)
        except Exception:
            logger.exception("endpoint pick failed")
            r = None
        self.stats["picks" if r else "no_pick"] += 1
        return r

    async def process(self, request_iterator, context):
        self.stats["streams"] += 1
        pick = None
        body = bytearray()
        routed = False
        try:
            async for raw in request_iterator:
                kind, d = decode_request(raw)
                if kind == "request_headers":
                    if d["end_of_stream"]:
                        pick, routed = self._route(b""), True
                        yield response(1, common_response(pick.headers() if pick else None, clear_route_cache=True))
                    else:
                        yield response(1, common_response())
                elif kind == "request_body":
                    body.extend(d["body"])
                    if d["end_of_stream"]:
                        if not routed:
                            pick, routed = self._route(bytes(body)), True
                        yield response(3, common_response(pick.headers() if pick else None, bytes(body), True,
                                                          clear_route_cache=True))
                elif kind == "response_headers":
                    yield response(2, common_response())
                elif kind == "response_body":
                    yield response(4, common_response(None, d["body"], d["end_of_stream"]))
                elif kind == "request_trailers":
                    yield response(5)
                elif kind == "response_trailers":
                    yield response(6)
        finally:
            if pick is not None:
                self.picker.release(pick)

    def handler(self):
        import grpc

        rpc = grpc.stream_stream_rpc_method_handler(self.process, request_deserializer=lambda b: b,
                                                    response_serializer=lambda b: b)
        return grpc.method_handlers_generic_handler(SERVICE, {METHOD: rpc})


async def serve(picker, host: str = "0.0.0.0", port: int = 9002):
    import grpc

    srv = grpc.aio.server()
    ep = ExtProcServer(picker)
    srv.add_generic_rpc_handlers((ep.handler(),))
    bound = srv.add_insecure_port(f"{host}:{port}")
    await srv.start()
    return srv, ep, bound

"""Prefill/decode disaggregated routing.

Per request: pick a prefill worker (``role_hint="prefill"``) and a decode
worker (``role_hint="decode"``) from breaker-filtered pools, resolve the
pair's protocol, forge a room id aligned to the prefill DP rank, then:

* concurrent topology: POST the prefill leg as a background task that is
  never cancelled (its KV push must complete even if the client leaves),
  open the decode stream with up to 3 pre-flight retries and backoff, relay
  it, and in ``finally`` await the prefill leg, score both legs on the
  breaker and release their in-flight blocks;
* serial-pull topology: POST prefill, wait for its JSON, extract the
  handoff, POST decode and relay it.

Flow of ``infera/router/disagg.py:66-1055``; the KV itself moves engine to
engine (here over NVLink by the engines), never through the router.
"""

from __future__ import annotations

import asyncio
import json
import logging
import random
import time

from fastapi.responses import JSONResponse, Response, StreamingResponse

from infera_b200.common.worker_pool import DisaggMode
from infera_b200.router.dp_routing import align_room_to_prefill_rank, dp_rank_header
from infera_b200.router.disagg_protocols import ProtocolError, resolve_protocol
from infera_b200.router.mixed import BaseRouter, forwardable
from infera_b200.router.transport import DATA, DONE, ERROR

logger = logging.getLogger(__name__)

DECODE_OPEN_RETRIES = 3
DECODE_OPEN_BACKOFF_S = 0.05


class DisaggRouter(BaseRouter):
    async def dispatch(self, body: dict, *, stream: bool, path: str = "/v1/chat/completions") -> Response:
        model = body.get("model")
        prefills = self.breaker.filter(self.pool.list_active(model=model, mode=DisaggMode.PREFILL))
        decodes = self.breaker.filter(self.pool.list_active(model=model, mode=DisaggMode.DECODE))
        if not prefills or not decodes:
            empty = "prefill" if not prefills else "decode"
            return JSONResponse({"error": f"no active {empty} worker for model={model!r}"}, status_code=503)
        pt, pblocks = self.policy.pick(prefills, body, role_hint="prefill")
        dt, dblocks = self.policy.pick(decodes, body, role_hint="decode")
        return await self.dispatch_pair(body, pt, pblocks, dt, dblocks, stream=stream, path=path)

    async def dispatch_pair(self, body, pt, pblocks, dt, dblocks, *, stream: bool, path: str) -> Response:
        p, d = pt.worker, dt.worker
        try:
            proto = resolve_protocol(p, d)
        except ProtocolError as e:
            return JSONResponse({"error": str(e)}, status_code=500)
        room = random.getrandbits(63)
        if getattr(proto, "pin_prefill_dp_rank", False):
            room = align_room_to_prefill_rank(room, pt)
        rid = proto.request_id_for(p, d, room)
        base = forwardable(body)
        hdr_p = dict(dp_rank_header(pt))
        hdr_d = dict(dp_rank_header(dt))
        if rid:
            hdr_p["X-Request-Id"] = rid
            hdr_d["X-Request-Id"] = rid
        self.policy.on_request_started(pt.route_key, pblocks)
        self.policy.on_request_started(dt.route_key, dblocks)
        if proto.topology == "serial-pull":
            return await self._serial(proto, base, pt, pblocks, dt, dblocks, room, hdr_p, hdr_d, stream, path)
        return await self._concurrent(proto, base, pt, pblocks, dt, dblocks, room, hdr_p, hdr_d, stream, path)

    async def _prefill_leg(self, pt, body, headers, path) -> tuple[int, bytes]:
        t0 = time.monotonic()
        status, raw = 0, b""
        try:
            async for kind, st, data in self.transport.stream(pt.worker, path, body, headers):
                if kind == DATA:
                    raw += data
                    status = st or 200
                elif kind == ERROR:
                    status, raw = st or 0, data
                    break
        finally:
            if self.metrics is not None:
                self.metrics.pd_leg("prefill", time.monotonic() - t0)
        return status, raw

    async def _open_decode(self, dt, body, headers, path):
        last = (502, b"")
        for attempt in range(DECODE_OPEN_RETRIES):
            agen = self.transport.stream(dt.worker, path, body, headers)
            try:
                kind, st, d0 = await agen.__anext__()
            except StopAsyncIteration:
                kind, st, d0 = DONE, 200, b""
            if kind == DATA:
                return agen, d0, None
            await agen.aclose()
            last = (st or 502, d0)
            await asyncio.sleep(DECODE_OPEN_BACKOFF_S * (2 ** attempt))
        return None, None, last

    async def _concurrent(self, proto, base, pt, pblocks, dt, dblocks, room, hdr_p, hdr_d, stream, path):
        pbody = proto.annotate_prefill(base, pt.worker, dt.worker, room)
        dbody = proto.annotate_decode(base, pt.worker, dt.worker, room, None)
        dbody["stream"] = stream
        ptask = asyncio.ensure_future(self._prefill_leg(pt, pbody, hdr_p, path))
        agen, d0, err = await self._open_decode(dt, dbody, hdr_d, path)

        async def finish():
            try:
                pst, _ = await asyncio.shield(ptask)
            except Exception:
                pst = 0
            self.breaker.record_outcome(pt.worker.worker_id, pst if pst else 0)
            self.policy.on_request_finished(pt.route_key, pblocks)
            self.policy.on_request_finished(dt.route_key, dblocks)

        if agen is None:
            self.breaker.record_failure(dt.worker.worker_id, err[0])
            await finish()
            return JSONResponse({"error": f"decode worker {dt.worker.worker_id} failed to open",
                                 "raw": err[1][:300].decode("utf-8", "replace")}, status_code=err[0])
        self.breaker.record_success(dt.worker.worker_id)
        if not stream:
            raw = d0
            async for k, _s, d in agen:
                if k == DATA:
                    raw += d
            await finish()
            try:
                return JSONResponse(json.loads(raw))
            except ValueError:
                return Response(raw, media_type="application/json")

        async def relay():
            t0 = time.monotonic()
            try:
                yield d0
                async for k, _s, d in agen:
                    if k == DATA:
                        yield d
                    elif k == ERROR:
                        yield f'data: {{"error":"decode worker {dt.worker.worker_id} failed mid-stream"}}\n\n'.encode()
                        break
                    else:
                        break
            finally:
                if self.metrics is not None:
                    self.metrics.pd_leg("decode", time.monotonic() - t0)
                await finish()

        return StreamingResponse(relay(), media_type="text/event-stream")

    async def _serial(self, proto, base, pt, pblocks, dt, dblocks, room, hdr_p, hdr_d, stream, path):
        pbody = proto.annotate_prefill(base, pt.worker, dt.worker, room)
        pst, raw = await self._prefill_leg(pt, pbody, hdr_p, path)
        self.breaker.record_outcome(pt.worker.worker_id, pst)
        if pst >= 400 or pst == 0:
            self.policy.on_request_finished(pt.route_key, pblocks)
            self.policy.on_request_finished(dt.route_key, dblocks)
            return JSONResponse({"error": f"prefill worker {pt.worker.worker_id} failed"},
                                status_code=pst if pst >= 400 else 502)
        try:
            handoff = proto.extract_handoff(json.loads(raw))
        except ValueError:
            handoff = {}
        self.policy.on_request_finished(pt.route_key, pblocks)
        dbody = proto.annotate_decode(base, pt.worker, dt.worker, room, handoff)
        dbody["stream"] = stream
        agen, d0, err = await self._open_decode(dt, dbody, hdr_d, path)
        if agen is None:
            self.breaker.record_failure(dt.worker.worker_id, err[0])
            self.policy.on_request_finished(dt.route_key, dblocks)
            return JSONResponse({"error": f"decode worker {dt.worker.worker_id} failed to open"}, status_code=err[0])

        async def relay():
            try:
                yield d0
                async for k, _s, d in agen:
                    if k == DATA:
                        yield d
                    else:
                        break
            finally:
                self.policy.on_request_finished(dt.route_key, dblocks)

        if not stream:
            out = d0
            async for k, _s, d in agen:
                if k == DATA:
                    out += d
            self.policy.on_request_finished(dt.route_key, dblocks)
            return Response(out, media_type="application/json")
        return StreamingResponse(relay(), media_type="text/event-stream")

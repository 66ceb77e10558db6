"""Aggregated (mixed-role) routing with failover, breaker and migration.

``dispatch``: up to ``1 + request_max_retries`` attempts; each picks among
the active mixed workers not yet tried (after the breaker's filter). An
attempt that fails before the first byte raises :class:`Retry` and the loop
moves on; once the first data event is in hand the response is committed
and streamed. A stream that breaks later, or a worker that hands the request
back while draining, continues on another worker through
:class:`~infera_b200.router.migration.MigrationState` (when
``migration_limit > 0``). In-flight block refcounts go to the policy on
start / finish. Flow of ``infera/router/mixed.py:75-523``.
"""

from __future__ import annotations

import json
import logging
from typing import AsyncIterator

from fastapi.responses import JSONResponse, Response, StreamingResponse

from infera_b200.common.worker_pool import DisaggMode
from infera_b200.router.breaker import CircuitBreaker, is_worker_fault
from infera_b200.router.cache_control import parse_cache_hints
from infera_b200.router.dp_routing import dp_rank_header
from infera_b200.router.engine_priority import inject_engine_priority
from infera_b200.router.migration import MigrationState, as_chat_chunk
from infera_b200.router.transport import DATA, DONE, DRAINING_NOTICE, ERROR, HttpTransport

logger = logging.getLogger(__name__)


class Retry(Exception):
    def __init__(self, response: Response, status: int):
        super().__init__(status)
        self.response = response
        self.status = status


def forwardable(body: dict) -> dict:
    return {k: v for k, v in body.items() if not k.startswith("_infera")}


class BaseRouter:
    def __init__(self, pool, policy, *, transport=None, breaker: CircuitBreaker | None = None,
                 request_max_retries: int = 1, migration_limit: int = 0, metrics=None):
        self.pool = pool
        self.policy = policy
        self.transport = transport or HttpTransport()
        self.breaker = breaker or CircuitBreaker()
        self.request_max_retries = request_max_retries
        self.migration_limit = migration_limit
        self.metrics = metrics

    async def dispatch(self, body: dict, *, stream: bool, path: str = "/v1/chat/completions") -> Response:
        raise NotImplementedError

    async def aclose(self) -> None:
        await self.transport.aclose()


class MixedRouter(BaseRouter):
    mode = DisaggMode.MIXED

    async def dispatch(self, body: dict, *, stream: bool, path: str = "/v1/chat/completions") -> Response:
        model = body.get("model")
        hints = body.get("_infera_cache_hints") or parse_cache_hints(body)
        body["_infera_cache_hints"] = hints
        tried: set[str] = set()
        last: Response | None = None
        for _ in range(1 + self.request_max_retries):
            cands = [w for w in self.pool.list_active(model=model, mode=self.mode) if w.worker_id not in tried]
            cands = self.breaker.filter(cands)
            if not cands:
                break
            target, blocks = self.policy.pick(cands, body)
            tried.add(target.worker.worker_id)
            try:
                resp = await self._attempt(target, blocks, body, hints, path, stream)
                if resp.status_code < 400:
                    self.breaker.record_success(target.worker.worker_id)
                else:
                    self.breaker.record_failure(target.worker.worker_id, resp.status_code)
                return resp
            except Retry as r:
                self.breaker.record_failure(target.worker.worker_id, r.status)
                last = r.response
                logger.info("failover: %s failed before first byte (%d tried)", target.worker.worker_id, len(tried))
        if last is not None:
            return last
        return JSONResponse({"error": f"no active {self.mode.value} worker for model={model!r}"}, status_code=503)

    async def _attempt(self, target, blocks, body, hints, path, stream) -> Response:
        worker = target.worker
        fwd = forwardable(inject_engine_priority(body, hints, worker.engine))
        if stream and self.migration_limit > 0:
            fwd["return_token_ids"] = True
        headers = dp_rank_header(target)
        self.policy.on_request_started(target.route_key, blocks)
        agen = self.transport.stream(worker, path, fwd, headers)
        try:
            kind, status, data0 = await agen.__anext__()
        except StopAsyncIteration:
            kind, status, data0 = DONE, 200, b""
        if kind != DATA:
            await agen.aclose()
            self.policy.on_request_finished(target.route_key, blocks)
            code = status if status and status >= 400 else 502
            raise Retry(JSONResponse({"error": f"worker {worker.worker_id} failed before first token",
                                      "raw": (data0 or b"")[:500].decode("utf-8", "replace")},
                                     status_code=code), code)
        if not stream:
            rest = b""
            async for k, st, d in agen:
                if k == DATA:
                    rest += d
            self.policy.on_request_finished(target.route_key, blocks)
            raw = data0 + rest
            try:
                obj = json.loads(raw)
                from infera_b200.router.token_ids import strip_token_ids

                if "return_token_ids" not in body:
                    strip_token_ids(obj)
                return JSONResponse(obj, status_code=status or 200)
            except ValueError:
                return Response(raw, status_code=status or 200, media_type="application/json")
        state = MigrationState(body, self.migration_limit, path) if self.migration_limit > 0 else None
        return StreamingResponse(self._relay(agen, data0, target, blocks, state, path),
                                 media_type="text/event-stream")

    async def _relay(self, agen, data0: bytes, target, blocks, state, path) -> AsyncIterator[bytes]:
        cur, cur_t, cur_b = agen, target, blocks

        def passthrough(ev):
            return state.observe(ev) if state is not None else ev

        transform = passthrough
        try:
            if data0:
                yield transform(data0)
            while True:
                reason = "stream_broken"
                async for k, _st, d in cur:
                    if k == DATA:
                        if d:
                            yield transform(d)
                    elif k == ERROR:
                        if d.startswith(DRAINING_NOTICE.encode()):
                            reason = "worker_draining"
                        break
                    else:
                        return
                resumed = None
                if state is not None and state.can_migrate():
                    resumed = await self._resume_elsewhere(state, cur_t, path, reason)
                if resumed is None:
                    what = "is shutting down" if reason == "worker_draining" else "failed"
                    yield f'data: {{"error":"worker {cur_t.worker.worker_id} {what} mid-stream"}}\n\n'.encode()
                    return
                nxt, nt, nb, reshape = resumed
                self.policy.on_request_finished(cur_t.route_key, cur_b)
                cur, cur_t, cur_b = nxt, nt, nb
                if reshape:
                    transform = lambda ev: as_chat_chunk(passthrough(ev))  # noqa: E731
                else:
                    transform = passthrough
        finally:
            self.policy.on_request_finished(cur_t.route_key, cur_b)

    async def _resume_elsewhere(self, state: MigrationState, failed, path, reason):
        cont = state.next_continuation()
        model = cont.body.get("model")
        cands = [w for w in self.pool.list_active(model=model, mode=self.mode)
                 if w.worker_id != failed.worker.worker_id]
        cands = self.breaker.filter(cands)
        while cands:
            target, blocks = self.policy.pick(cands, cont.body)
            cands = [w for w in cands if w.worker_id != target.worker.worker_id]
            self.policy.on_request_started(target.route_key, blocks)
            agen = self.transport.stream(target.worker, cont.path, cont.body, dp_rank_header(target))
            try:
                kind, status, d0 = await agen.__anext__()
            except StopAsyncIteration:
                kind, status, d0 = DONE, 200, b""
            if kind == DATA:
                if self.metrics is not None:
                    self.metrics.migrations(reason)

                async def chain(first=d0, rest=agen):
                    yield DATA, 200, first
                    async for item in rest:
                        yield item

                return chain(), target, blocks, cont.reshape_to_chat
            await agen.aclose()
            self.policy.on_request_finished(target.route_key, blocks)
            self.breaker.record_failure(target.worker.worker_id, status)
        return None

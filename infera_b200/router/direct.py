"""Gateway-directed routing: the gateway (GAIE endpoint picker) already
chose the worker(s) and names them in ``x-worker-instance-id`` (and
``x-prefill-instance-id`` for PD); no failover
(``infera/router/direct.py:30-101``)."""

from __future__ import annotations

from fastapi.responses import JSONResponse, Response

from infera_b200.common.worker_pool import DisaggMode
from infera_b200.router.disagg import DisaggRouter
from infera_b200.router.mixed import BaseRouter, MixedRouter, Retry
from infera_b200.router.policy.target import RouteTarget

WORKER_HEADER = "x-worker-instance-id"
PREFILL_HEADER = "x-prefill-instance-id"


class DirectRouter(BaseRouter):
    def __init__(self, pool, policy, **kw):
        kw["request_max_retries"] = 0
        super().__init__(pool, policy, **kw)
        shared = dict(transport=self.transport, breaker=self.breaker, request_max_retries=0,
                      migration_limit=self.migration_limit, metrics=self.metrics)
        self.mixed = MixedRouter(pool, policy, **shared)
        self.disagg = DisaggRouter(pool, policy, **shared)

    async def dispatch(self, body: dict, *, stream: bool, path: str = "/v1/chat/completions") -> Response:
        wid = body.get("_infera_direct_worker")
        pid = body.get("_infera_direct_prefill")
        if not wid:
            return JSONResponse({"error": f"missing {WORKER_HEADER} header"}, status_code=400)
        w = self.pool.get(wid)
        if w is None:
            return JSONResponse({"error": f"unknown worker {wid!r}"}, status_code=404)
        if pid:
            p = self.pool.get(pid)
            if p is None:
                return JSONResponse({"error": f"unknown prefill worker {pid!r}"}, status_code=404)
            return await self.disagg.dispatch_pair(body, RouteTarget(p, p.dp_rank), [], RouteTarget(w, w.dp_rank),
                                                   [], stream=stream, path=path)
        if w.disagg_mode != DisaggMode.MIXED:
            return JSONResponse({"error": f"worker {wid!r} is {w.disagg_mode.value}; name a prefill worker too"},
                                status_code=400)
        t = RouteTarget(w, w.dp_rank)
        try:
            resp = await self.mixed._attempt(t, [], body, body.get("_infera_cache_hints"), path, stream)
        except Retry as r:  # no failover in direct mode: the gateway picked this worker
            self.breaker.record_failure(wid, r.status)
            return r.response
        self.breaker.record_success(wid)
        return resp

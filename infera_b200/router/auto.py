"""Per-request choice between aggregated and disaggregated routing.

If the model has both prefill and decode workers -> disaggregated; if it
has exactly one of the two PD pools and no mixed workers -> 503 naming the
empty pool; otherwise -> mixed. One breaker is shared
(``infera/router/auto.py:21-106``)."""

from __future__ import annotations

from fastapi.responses import JSONResponse, Response

from infera_b200.common.worker_pool import DisaggMode
from infera_b200.router.disagg import DisaggRouter
from infera_b200.router.mixed import BaseRouter, MixedRouter


class AutoRouter(BaseRouter):
    def __init__(self, pool, policy, **kw):
        super().__init__(pool, policy, **kw)
        shared = dict(transport=self.transport, breaker=self.breaker, request_max_retries=self.request_max_retries,
                      migration_limit=self.migration_limit, metrics=self.metrics)
        self.mixed = MixedRouter(pool, policy, **shared)
        self.disagg = DisaggRouter(pool, policy, **shared)

    async def dispatch(self, body: dict, *, stream: bool, path: str = "/v1/chat/completions") -> Response:
        model = body.get("model")
        p = self.pool.list_active(model=model, mode=DisaggMode.PREFILL)
        d = self.pool.list_active(model=model, mode=DisaggMode.DECODE)
        if p and d:
            return await self.disagg.dispatch(body, stream=stream, path=path)
        m = self.pool.list_active(model=model, mode=DisaggMode.MIXED)
        if (p or d) and not m:
            empty = "decode" if p else "prefill"
            return JSONResponse({"error": f"model {model!r} has {'prefill' if p else 'decode'} workers but no "
                                          f"active {empty} workers"}, status_code=503)
        return await self.mixed.dispatch(body, stream=stream, path=path)

"""HTTP(S) front for :class:`~infera_b200.common.k8s_client.FakeK8sClient`:
the Pod list and watch routes of the Kubernetes API, for running the
native router's Kubernetes discovery without a cluster (tests, the CPU
fleet).

    GET /api/v1/namespaces/{ns}/pods?labelSelector=...            -> PodList
    GET /api/v1/namespaces/{ns}/pods?watch=true&resourceVersion=N  -> JSON lines
        (events after N replayed first, then new ones; BOOKMARKs are not sent)

``require_token``: requests without ``Authorization: Bearer <token>`` get
401, as the API server answers a Pod without a service account.
"""

from __future__ import annotations

import asyncio
import json

from starlette.applications import Starlette
from starlette.requests import Request
from starlette.responses import JSONResponse, StreamingResponse
from starlette.routing import Route

from infera_b200.common.k8s_client import FakeK8sClient


def build_app(fake: FakeK8sClient, require_token: str | None = None) -> Starlette:
    async def pods(request: Request):
        if require_token is not None and request.headers.get("authorization") != f"Bearer {require_token}":
            return JSONResponse({"kind": "Status", "code": 401, "reason": "Unauthorized"}, status_code=401)
        ns = request.path_params["ns"]
        sel = request.query_params.get("labelSelector", "")
        if request.query_params.get("watch") not in ("true", "1"):
            return JSONResponse(await fake.list_pods(ns, sel))
        rv = request.query_params.get("resourceVersion", "0")

        async def stream():
            q: asyncio.Queue = asyncio.Queue()
            entry = (ns, sel, q)
            fake._watchers.append(entry)      # registered before the backlog is read: nothing falls between
            try:
                backlog = fake.events_since(ns, sel, rv)
                seen = {int(e["object"]["metadata"]["resourceVersion"]) for e in backlog}
                for ev in backlog:
                    yield (json.dumps(ev) + "\n").encode()
                while True:
                    try:
                        ev = await asyncio.wait_for(q.get(), timeout=30.0)
                    except asyncio.TimeoutError:
                        continue
                    if ev is None:
                        return
                    if int(ev["object"]["metadata"]["resourceVersion"]) in seen:
                        continue
                    yield (json.dumps(ev) + "\n").encode()
            finally:
                fake._watchers.remove(entry)

        return StreamingResponse(stream(), media_type="application/json")

    return Starlette(routes=[Route("/api/v1/namespaces/{ns}/pods", pods)])

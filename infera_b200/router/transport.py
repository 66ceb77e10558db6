"""How the router reaches a worker: normalized event streams.

Every transport yields ``(kind, status, data)`` tuples: ``kind`` is
``"data"`` (one SSE event or a unary body, bytes), ``"error"`` (the worker
failed; ``data`` says why, and starts with :data:`DRAINING_NOTICE` when the
worker is draining and hands the request back), or ``"done"``.

* :class:`HttpTransport` - httpx streaming POST to ``worker.url + path``;
* :class:`InProcessTransport` - calls a worker object living in the same
  process (tests, single-process fleets), with identical framing.
"""

from __future__ import annotations

from typing import AsyncIterator

import httpx

DATA, ERROR, DONE = "data", "error", "done"
DRAINING_NOTICE = "infera-worker-draining"


class HttpTransport:
    def __init__(self, client: httpx.AsyncClient | None = None):
        self.client = client or httpx.AsyncClient(
            timeout=httpx.Timeout(None, connect=60.0),
            limits=httpx.Limits(max_connections=None, max_keepalive_connections=4096))

    async def stream(self, worker, path: str, body: dict, headers: dict | None = None
                     ) -> AsyncIterator[tuple[str, int, bytes]]:
        url = worker.url + path
        try:
            async with self.client.stream("POST", url, json=body, headers=headers or {}) as resp:
                if resp.status_code >= 400:
                    raw = await resp.aread()
                    yield ERROR, resp.status_code, raw
                    return
                if not body.get("stream"):
                    raw = await resp.aread()
                    yield DATA, resp.status_code, raw
                    yield DONE, resp.status_code, b""
                    return
                buf = b""
                async for chunk in resp.aiter_bytes():
                    buf += chunk
                    while b"\n\n" in buf:
                        ev, buf = buf.split(b"\n\n", 1)
                        if not ev.strip():
                            continue
                        if ev.startswith(b"data: [DONE]"):
                            yield DATA, 200, ev + b"\n\n"
                            yield DONE, 200, b""
                            return
                        if DRAINING_NOTICE.encode() in ev and b'"error"' in ev:
                            yield ERROR, 503, DRAINING_NOTICE.encode()
                            return
                        yield DATA, 200, ev + b"\n\n"
                if buf.strip():
                    yield DATA, 200, buf
                # stream ended without [DONE]: a broken worker
                yield ERROR, 0, b"stream ended without [DONE]"
        except httpx.HTTPError as e:
            yield ERROR, 0, f"transport error: {e}".encode()

    async def get(self, worker, path: str) -> httpx.Response:
        return await self.client.get(worker.url + path)

    async def post(self, worker, path: str, body: dict | None = None) -> httpx.Response:
        return await self.client.post(worker.url + path, json=body or {})

    async def aclose(self) -> None:
        await self.client.aclose()


class InProcessTransport:
    """``workers[worker_id]`` must provide ``async handle(path, body, headers)``
    yielding the same (kind, status, data) tuples."""

    def __init__(self, workers: dict):
        self.workers = workers

    async def stream(self, worker, path, body, headers=None):
        w = self.workers.get(worker.worker_id)
        if w is None:
            yield ERROR, 0, b"no such worker"
            return
        async for item in w.handle(path, body, headers or {}):
            yield item

    async def get(self, worker, path):
        w = self.workers[worker.worker_id]
        return await w.get(path)

    async def post(self, worker, path, body=None):
        w = self.workers[worker.worker_id]
        return await w.post(path, body or {})

    async def aclose(self) -> None:
        return None


class RoutingTransport:
    """Picks a transport per worker from its record's ``request_transport``
    (``http`` by default; ``bus`` for workers behind a message bus)."""

    def __init__(self, http: HttpTransport | None = None, bus_client=None):
        self.http = http or HttpTransport()
        self.bus = bus_client

    def _for(self, worker):
        if getattr(worker, "request_transport", "http") == "bus":
            if self.bus is None:
                raise LookupError(f"worker {worker.worker_id} wants the bus transport but none is configured")
            return self.bus
        return self.http

    async def stream(self, worker, path, body, headers=None):
        try:
            t = self._for(worker)
        except LookupError as e:
            yield ERROR, 0, str(e).encode()
            return
        async for item in t.stream(worker, path, body, headers):
            yield item

    async def get(self, worker, path):
        return await self.http.get(worker, path)

    async def post(self, worker, path, body=None):
        return await self.http.post(worker, path, body)

    async def aclose(self) -> None:
        await self.http.aclose()

"""Request transport over a message bus (the reference's NATS path), with
an in-process bus.

Framing (``infera/common/nats_request.py:74-136``): the router publishes a
request on ``infera.req.<token>`` with a private reply subject; the worker
answers with frames whose headers carry ``rs-type`` (``data`` / ``done`` /
``error``) and ``rs-status``. The router gives up after ``idle_timeout`` s
without a frame (default 900) or ``max_duration`` s in total: it answers
504 and publishes ``infera.cancel.<token>`` (three times) so the worker
stops the work. Before sending, it asks ``infera.admit.<token>``: a worker
whose queued + running count is at its limit answers no and the router
answers 429 without queueing (the admission the reference does with a
JetStream work queue).

Worker side (:class:`BusRequestServer`): runs requests through a handler
(an async iterator of ``(kind, status, data)``, e.g. a proxy to the local
engine), at most ``max_concurrency`` at a time; ``drain`` stops admitting,
waits for queued and running requests and, after ``handback_after`` s,
ends the still-running streams with the draining notice so the router
migrates them.

:class:`InProcessBus` implements subjects, inboxes and request/reply in
one process (no NATS server exists on these machines); a NATS client with
the same four methods can replace it.
"""

from __future__ import annotations

import asyncio
import itertools
import json
import time
import uuid
from dataclasses import dataclass, field
from typing import AsyncIterator, Awaitable, Callable

from infera_b200.router.transport import DATA, DONE, DRAINING_NOTICE, ERROR

REQ = "infera.req."
CANCEL = "infera.cancel."
ADMIT = "infera.admit."
CANCEL_RESENDS = 3


@dataclass
class Msg:
    subject: str
    data: bytes = b""
    headers: dict = field(default_factory=dict)
    reply: str | None = None


class InProcessBus:
    def __init__(self) -> None:
        self._subs: dict[str, list[Callable[[Msg], Awaitable[None]]]] = {}
        self._ids = itertools.count()

    def new_inbox(self) -> str:
        return f"_INBOX.{uuid.uuid4().hex}"

    async def subscribe(self, subject: str, cb: Callable[[Msg], Awaitable[None]]) -> Callable[[], None]:
        self._subs.setdefault(subject, []).append(cb)

        def unsubscribe():
            lst = self._subs.get(subject, [])
            if cb in lst:
                lst.remove(cb)

        return unsubscribe

    async def publish(self, subject: str, data: bytes = b"", headers: dict | None = None,
                      reply: str | None = None) -> None:
        for cb in list(self._subs.get(subject, [])):
            asyncio.get_running_loop().create_task(cb(Msg(subject, data, dict(headers or {}), reply)))

    async def request(self, subject: str, data: bytes = b"", timeout: float = 5.0) -> Msg:
        inbox = self.new_inbox()
        fut = asyncio.get_running_loop().create_future()

        async def on_reply(m: Msg):
            if not fut.done():
                fut.set_result(m)

        unsub = await self.subscribe(inbox, on_reply)
        try:
            await self.publish(subject, data, reply=inbox)
            return await asyncio.wait_for(fut, timeout)
        finally:
            unsub()


def _frame_headers(kind: str, status: int) -> dict:
    return {"rs-type": kind, "rs-status": str(status)}


REQUEST_STREAM = "INFERA_REQUESTS"
HDR_INBOX = "infera-inbox"


def request_durable(token: str) -> str:
    """Durable JetStream consumer of one worker's request subject."""
    return f"infera-req-{token}"


class BusRequestClient:
    """Router side; ``stream`` has the router transports' interface.

    ``jetstream=True``: requests go through the ``INFERA_REQUESTS``
    work-queue stream (one durable consumer per worker; the reply inbox rides
    in a header because a stream-delivered message's reply subject is its
    ack subject), and admission is the worker consumer's pending count
    against ``max_pending`` instead of an admit request."""

    def __init__(self, bus, idle_timeout: float = 900.0, max_duration: float | None = None,
                 admit_timeout: float = 2.0, jetstream: bool = False, max_pending: int = 64):
        self.bus = bus
        self.idle_timeout = idle_timeout
        self.max_duration = max_duration
        self.admit_timeout = admit_timeout
        self.jetstream = jetstream
        self.max_pending = max_pending
        self._js = None
        self.stats = {"requests": 0, "rejected": 0, "timeouts": 0, "cancels_sent": 0}

    async def _jetstream(self):
        if self._js is None:
            from infera_b200.common.jetstream import JetStream

            js = JetStream(self.bus)
            await js.add_stream(REQUEST_STREAM, [REQ + ">"], retention="workqueue")
            self._js = js
        return self._js

    @staticmethod
    def token(worker) -> str:
        return str(worker.worker_id).replace(".", "_").replace(":", "_")

    async def admit(self, worker) -> bool:
        if self.jetstream:
            from infera_b200.common.jetstream import JetStreamError

            js = await self._jetstream()
            try:
                info = await js.consumer_info(REQUEST_STREAM, request_durable(self.token(worker)))
            except (JetStreamError, asyncio.TimeoutError):
                return False      # the worker has not attached its consumer: not serving
            return int(info.get("num_pending", 0)) < self.max_pending
        try:
            m = await self.bus.request(ADMIT + self.token(worker), b"", timeout=self.admit_timeout)
        except asyncio.TimeoutError:
            return False
        return bool(json.loads(m.data or b"{}").get("ok"))

    async def _cancel(self, worker, rid: str) -> None:
        for _ in range(CANCEL_RESENDS):
            await self.bus.publish(CANCEL + self.token(worker), rid.encode())
            self.stats["cancels_sent"] += 1

    async def stream(self, worker, path: str, body: dict, headers: dict | None = None
                     ) -> AsyncIterator[tuple[str, int, bytes]]:
        self.stats["requests"] += 1
        if not await self.admit(worker):
            self.stats["rejected"] += 1
            yield ERROR, 429, b"worker at its admission limit"
            return
        rid = uuid.uuid4().hex
        inbox = self.bus.new_inbox()
        q: asyncio.Queue = asyncio.Queue()

        async def on_frame(m: Msg):
            q.put_nowait(m)

        unsub = await self.bus.subscribe(inbox, on_frame)
        t0 = time.monotonic()
        try:
            payload = json.dumps({"path": path, "body": body, "headers": headers or {}}).encode()
            if self.jetstream:
                js = await self._jetstream()
                await js.publish(REQ + self.token(worker), payload, headers={"rid": rid, HDR_INBOX: inbox})
            else:
                await self.bus.publish(REQ + self.token(worker), payload, headers={"rid": rid}, reply=inbox)
            while True:
                wait = self.idle_timeout
                if self.max_duration is not None:
                    wait = min(wait, max(0.0, self.max_duration - (time.monotonic() - t0)))
                try:
                    m = await asyncio.wait_for(q.get(), wait)
                except asyncio.TimeoutError:
                    self.stats["timeouts"] += 1
                    await self._cancel(worker, rid)
                    yield ERROR, 504, b"worker timed out"
                    return
                kind = m.headers.get("rs-type", DATA)
                status = int(m.headers.get("rs-status", "200"))
                yield kind, status, m.data
                if kind in (DONE, ERROR):
                    return
        finally:
            unsub()


Handler = Callable[[str, dict, dict], AsyncIterator[tuple[str, int, bytes]]]


class BusRequestServer:
    """Worker side: admission, bounded concurrency, cancel, drain, hand-back."""

    def __init__(self, bus, worker_token: str, handler: Handler, max_concurrency: int = 256,
                 max_pending: int = 1024, migratable: Callable[[dict], bool] | None = None,
                 jetstream: bool = False, fetch_batch: int = 8):
        self.bus = bus
        # jetstream: pull this worker's requests from its durable consumer on
        # the INFERA_REQUESTS work queue (each is acked when taken)
        self.jetstream = jetstream
        self.fetch_batch = fetch_batch
        self._pull: asyncio.Task | None = None
        self.token = worker_token
        self.handler = handler
        self.max_concurrency = max_concurrency
        self.max_pending = max_pending
        self.migratable = migratable or (lambda body: bool(body.get("stream")))
        self._sem = asyncio.Semaphore(max_concurrency)
        self._tasks: dict[str, tuple[asyncio.Task, dict, str]] = {}  # rid -> (task, body, reply subject)
        self._queued = 0
        self.draining = False
        self._unsubs: list = []
        self.stats = {"served": 0, "refused": 0, "cancelled": 0, "handed_back": 0}

    @property
    def inflight(self) -> int:
        return len(self._tasks)

    async def start(self) -> None:
        if self.jetstream:
            from infera_b200.common.jetstream import JetStream

            js = JetStream(self.bus)
            await js.add_stream(REQUEST_STREAM, [REQ + ">"], retention="workqueue")
            await js.add_consumer(REQUEST_STREAM, durable=request_durable(self.token), filter_subject=REQ + self.token)
            self._pull = asyncio.get_running_loop().create_task(self._pull_loop(js))
        else:
            self._unsubs.append(await self.bus.subscribe(REQ + self.token, self._on_request))
        self._unsubs.append(await self.bus.subscribe(CANCEL + self.token, self._on_cancel))
        self._unsubs.append(await self.bus.subscribe(ADMIT + self.token, self._on_admit))

    async def _pull_loop(self, js) -> None:
        durable = request_durable(self.token)
        while True:
            if self.draining:
                await asyncio.sleep(0.05)   # leave queued requests to the stream (and other workers' retries)
                continue
            try:
                msgs = await js.fetch(REQUEST_STREAM, durable, batch=self.fetch_batch, expires_s=1.0)
            except asyncio.CancelledError:
                raise
            except Exception:
                await asyncio.sleep(0.2)
                continue
            for jm in msgs:
                await js.ack(jm)
                await self._on_request(Msg(jm.subject, jm.data, jm.headers, jm.headers.get(HDR_INBOX)))

    async def stop(self) -> None:
        if self._pull is not None:
            self._pull.cancel()
            try:
                await self._pull
            except (asyncio.CancelledError, Exception):
                pass
            self._pull = None
        for u in self._unsubs:
            u()
        self._unsubs.clear()

    async def _on_admit(self, m: Msg) -> None:
        ok = not self.draining and self.inflight < self.max_pending
        if m.reply:
            await self.bus.publish(m.reply, json.dumps({"ok": ok, "pending": self.inflight}).encode())

    async def _on_cancel(self, m: Msg) -> None:
        ent = self._tasks.get(m.data.decode())
        if ent is not None and not ent[0].done():
            ent[0].cancel()
            self.stats["cancelled"] += 1

    async def _on_request(self, m: Msg) -> None:
        rid = m.headers.get("rid") or uuid.uuid4().hex
        if rid in self._tasks:
            return  # duplicate delivery
        if self.draining or self.inflight >= self.max_pending:
            self.stats["refused"] += 1
            status = 503 if self.draining else 429
            msg = DRAINING_NOTICE if self.draining else "worker at its admission limit"
            await self.bus.publish(m.reply, msg.encode(), _frame_headers(ERROR, status))
            return
        req = json.loads(m.data)
        task = asyncio.get_running_loop().create_task(self._serve(rid, req, m.reply))
        self._tasks[rid] = (task, req.get("body") or {}, m.reply)

    async def _serve(self, rid: str, req: dict, reply: str) -> None:
        try:
            async with self._sem:
                async for kind, status, data in self.handler(req["path"], req.get("body") or {},
                                                             req.get("headers") or {}):
                    await self.bus.publish(reply, data, _frame_headers(kind, status))
                    if kind in (DONE, ERROR):
                        break
                else:
                    await self.bus.publish(reply, b"", _frame_headers(DONE, 200))
            self.stats["served"] += 1
        except asyncio.CancelledError:
            pass
        finally:
            self._tasks.pop(rid, None)

    async def drain(self, timeout: float = 30.0, handback_after: float | None = None) -> bool:
        """Refuse new work, wait for queued + running; hand back streams
        still running after ``handback_after`` s. True if drained cleanly."""
        self.draining = True
        t0 = time.monotonic()
        handed = False
        while self._tasks:
            el = time.monotonic() - t0
            if handback_after is not None and el >= handback_after and not handed:
                handed = True
                for rid, (task, body, reply) in list(self._tasks.items()):
                    if self.migratable(body):
                        task.cancel()
                        self.stats["handed_back"] += 1
                        # the router sees the notice and migrates the stream
                        await self.bus.publish(reply, DRAINING_NOTICE.encode(), _frame_headers(ERROR, 503))
            if el >= timeout:
                return False
            await asyncio.sleep(0.01)
        return True


def local_http_handler(base_url: str, client=None) -> Handler:
    """Worker side of the bus transport: forward each request to this
    worker's own OpenAI HTTP server and relay its frames (the same SSE
    framing and error mapping as the router's HTTP transport)."""
    from infera_b200.router.transport import HttpTransport

    http = HttpTransport(client)

    class _Local:
        url = base_url.rstrip("/")

    async def handler(path: str, body: dict, headers: dict):
        async for item in http.stream(_Local, path, body, headers):
            yield item

    return handler

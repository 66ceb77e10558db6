"""Core NATS client over the NATS text protocol, with the message-bus
interface of :class:`infera_b200.common.request_transport.InProcessBus`
(``new_inbox`` / ``subscribe`` / ``publish`` / ``request``), so the request
transport and the KV-event relay run over a real NATS server.

Protocol (the public NATS client protocol): the server opens with
``INFO {json}``; the client sends ``CONNECT {json}`` (headers and
no-responders enabled) and ``PING``, and is connected at the ``PONG``.
``SUB <subject> <sid>`` / ``UNSUB <sid>`` manage subscriptions;
``PUB <subject> [reply] <n>`` and ``HPUB <subject> [reply] <hdr> <total>``
(a ``NATS/1.0`` header block, then the payload) publish; the server
delivers ``MSG <subject> <sid> [reply] <n>`` / ``HMSG ...`` and pings,
answered with ``PONG``. Requests use one wildcard inbox subscription
(``_INBOX.<id>.*``) and a token per request; a ``503`` status header (no
responders) resolves the request with an empty message.

Reference counterpart: the reference's request and KV-event paths over
NATS use the nats-py client (``infera/common/nats_request.py``,
``infera/kv/nats_bus.py``); that library is not available here, so this is
the protocol client itself (core NATS; JetStream admission is replaced by
the ``infera.admit.<token>`` request the bus transport already makes).
"""

from __future__ import annotations

import asyncio
import itertools
import json
import logging
import uuid
from typing import Awaitable, Callable
from urllib.parse import urlparse

from infera_b200.common.request_transport import Msg

log = logging.getLogger(__name__)


def parse_headers(block: bytes) -> dict:
    """``NATS/1.0[ status[ description]]`` then ``Key: Value`` lines; the
    status (if any) is returned under ``"status"``."""
    lines = block.decode("utf-8", "replace").split("\r\n")
    out: dict = {}
    first = lines[0] if lines else ""
    if first.startswith("NATS/1.0"):
        rest = first[len("NATS/1.0"):].strip()
        if rest:
            out["status"] = rest.split(" ", 1)[0]
    for ln in lines[1:]:
        if not ln:
            continue
        k, _, v = ln.partition(":")
        out[k.strip()] = v.strip()
    return out


def encode_headers(headers: dict) -> bytes:
    return ("NATS/1.0\r\n" + "".join(f"{k}: {v}\r\n" for k, v in headers.items()) + "\r\n").encode()


class NatsBus:
    def __init__(self, url: str = "nats://127.0.0.1:4222", name: str = "infera-b200"):
        u = urlparse(url if "://" in url else "nats://" + url)
        self.host, self.port = u.hostname or "127.0.0.1", u.port or 4222
        self.name = name
        self.server_info: dict = {}
        self._r: asyncio.StreamReader | None = None
        self._w: asyncio.StreamWriter | None = None
        self._subs: dict[int, Callable[[Msg], Awaitable[None]]] = {}
        self._sids = itertools.count(1)
        self._tokens = itertools.count(1)
        self._inbox = f"_INBOX.{uuid.uuid4().hex}"
        self._resp: dict[str, asyncio.Future] = {}
        self._resp_sid: int | None = None
        self._reader: asyncio.Task | None = None
        self._tasks: set[asyncio.Task] = set()
        self.closed = False

    # ------------------------------------------------------------------ connection
    async def connect(self, timeout: float = 5.0) -> "NatsBus":
        self._r, self._w = await asyncio.wait_for(asyncio.open_connection(self.host, self.port), timeout)
        line = await asyncio.wait_for(self._r.readline(), timeout)
        if not line.startswith(b"INFO "):
            raise ConnectionError(f"not a NATS server: {line[:80]!r}")
        self.server_info = json.loads(line[5:])
        opts = {"verbose": False, "pedantic": False, "headers": True, "no_responders": True, "protocol": 1,
                "lang": "python", "version": "infera-b200", "name": self.name}
        self._w.write(b"CONNECT " + json.dumps(opts).encode() + b"\r\nPING\r\n")
        await self._w.drain()
        while True:
            ln = await asyncio.wait_for(self._r.readline(), timeout)
            if not ln:
                raise ConnectionError("NATS server closed the connection during the handshake")
            if ln.startswith(b"PONG"):
                break
            if ln.startswith(b"-ERR"):
                raise ConnectionError(ln.decode().strip())
        self._reader = asyncio.get_running_loop().create_task(self._read_loop())
        return self

    async def close(self) -> None:
        self.closed = True
        if self._reader is not None:
            self._reader.cancel()
        if self._w is not None:
            self._w.close()
            try:
                await self._w.wait_closed()
            except Exception:
                pass

    async def _read_loop(self) -> None:
        r = self._r
        try:
            while True:
                line = await r.readline()
                if not line:
                    break
                if line.startswith(b"MSG "):
                    parts = line[4:].split()
                    subject, sid = parts[0].decode(), int(parts[1])
                    reply = parts[2].decode() if len(parts) == 4 else None
                    n = int(parts[-1])
                    data = (await r.readexactly(n + 2))[:n]
                    self._deliver(sid, Msg(subject, data, {}, reply))
                elif line.startswith(b"HMSG "):
                    parts = line[5:].split()
                    subject, sid = parts[0].decode(), int(parts[1])
                    reply = parts[2].decode() if len(parts) == 5 else None
                    hl, total = int(parts[-2]), int(parts[-1])
                    block = (await r.readexactly(total + 2))[:total]
                    self._deliver(sid, Msg(subject, block[hl:], parse_headers(block[:hl]), reply))
                elif line.startswith(b"PING"):
                    self._w.write(b"PONG\r\n")
                elif line.startswith(b"-ERR"):
                    log.warning("nats: %s", line.decode().strip())
                # PONG, +OK and INFO updates need no action
        except (asyncio.CancelledError, asyncio.IncompleteReadError, ConnectionError):
            pass

    def _deliver(self, sid: int, m: Msg) -> None:
        cb = self._subs.get(sid)
        if cb is None:
            return
        t = asyncio.get_running_loop().create_task(cb(m))
        self._tasks.add(t)
        t.add_done_callback(self._tasks.discard)

    # ------------------------------------------------------------------ bus interface
    def new_inbox(self) -> str:
        return f"_INBOX.{uuid.uuid4().hex}"

    async def subscribe(self, subject: str, cb: Callable[[Msg], Awaitable[None]]) -> Callable[[], None]:
        sid = next(self._sids)
        self._subs[sid] = cb
        self._w.write(f"SUB {subject} {sid}\r\n".encode())
        await self._w.drain()

        def unsubscribe() -> None:
            if self._subs.pop(sid, None) is not None and not self.closed:
                self._w.write(f"UNSUB {sid}\r\n".encode())

        return unsubscribe

    async def publish(self, subject: str, data: bytes = b"", headers: dict | None = None,
                      reply: str | None = None) -> None:
        rp = f" {reply}" if reply else ""
        if headers:
            hb = encode_headers(headers)
            self._w.write(f"HPUB {subject}{rp} {len(hb)} {len(hb) + len(data)}\r\n".encode() + hb + data + b"\r\n")
        else:
            self._w.write(f"PUB {subject}{rp} {len(data)}\r\n".encode() + data + b"\r\n")
        await self._w.drain()

    async def request(self, subject: str, data: bytes = b"", timeout: float = 5.0) -> Msg:
        if self._resp_sid is None:
            self._resp_sid = -1   # set before the await: concurrent first requests subscribe once
            unsub = await self.subscribe(self._inbox + ".*", self._on_response)
            self._resp_sid = 0
            self._resp_unsub = unsub
        token = str(next(self._tokens))
        fut = asyncio.get_running_loop().create_future()
        self._resp[token] = fut
        try:
            await self.publish(subject, data, reply=f"{self._inbox}.{token}")
            return await asyncio.wait_for(fut, timeout)
        finally:
            self._resp.pop(token, None)

    async def _on_response(self, m: Msg) -> None:
        fut = self._resp.get(m.subject.rsplit(".", 1)[-1])
        if fut is not None and not fut.done():
            fut.set_result(m)

"""Async client of the KV tier daemon.

``connect(shared_arena=True)`` negotiates the arena and maps its memfd, after
which GETs return arena offsets and the bytes are read in place with the
seqlock protocol (a rewrite between lookup and read yields a miss instead of
torn data); ``set_lease`` / ``commit_set`` let the caller fill a slot in
place. :class:`KvdPrefetchClient` is the router's fire-and-forget
``PREFETCH_HINT`` sender behind ``POST /v1/cache/prewarm``.
"""

from __future__ import annotations

import asyncio
import socket

from infera_b200.kvd import wire as W
from infera_b200.kvd.shared_arena import ArenaView


class KvdClient:
    def __init__(self, path: str, client_id: str = "infera-b200"):
        self.path = path
        self.client_id = client_id
        self.reader = None
        self.writer = None
        self.arena: ArenaView | None = None
        self._lock = asyncio.Lock()

    def _handshake(self, shared_arena: bool):
        """Blocking HELLO on a plain socket: reads exactly the ack frame, then
        the one-byte message that carries the arena fd, so that no buffered
        reader can swallow the ancillary data."""
        sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        sock.connect(self.path)
        sock.sendall(W.encode(W.Hello(self.client_id, 1, shared_arena)))

        def exactly(n: int) -> bytes:
            buf = b""
            while len(buf) < n:
                chunk = sock.recv(n - len(buf))
                if not chunk:
                    raise ConnectionError("kvd closed the connection during HELLO")
                buf += chunk
            return buf

        ack = W.decode_body(exactly(int.from_bytes(exactly(4), "big")))
        fd = None
        if shared_arena and ack.shared_arena is not None:
            _m, fds, _f, _a = socket.recv_fds(sock, 1, 1)
            fd = fds[0]
        sock.setblocking(False)
        return sock, ack, fd

    async def connect(self, shared_arena: bool = False) -> None:
        loop = asyncio.get_running_loop()
        sock, ack, fd = await loop.run_in_executor(None, self._handshake, shared_arena)
        self.reader, self.writer = await asyncio.open_unix_connection(sock=sock)
        if fd is not None:
            size, slot, _pid = ack.shared_arena
            self.arena = ArenaView(fd, size, slot)

    async def _call(self, msg):
        async with self._lock:
            await W.write_frame(self.writer, msg)
            return await W.read_frame(self.reader)

    async def get_shared(self, key: bytes):
        """(payload offset in the arena, size, version) of a value held in the
        shared arena; None when it is not (missing, or served inline)."""
        r = await self._call(W.Get(key))
        if isinstance(r, W.GetSharedResponse):
            return r.slot_offset, r.size, r.version
        return None

    async def get(self, key: bytes) -> bytes | None:
        r = await self._call(W.Get(key))
        if isinstance(r, W.GetSharedResponse):
            return self.arena.read(r.slot_offset, r.version)
        return r.value

    async def batch_get(self, keys: list[bytes]) -> list[bytes | None]:
        r = await self._call(W.BatchGet(keys))
        if isinstance(r, W.BatchGetSharedResponse):
            return [None if e is None else self.arena.read(e[0], e[2]) for e in r.entries]
        return r.values

    async def set(self, key: bytes, value: bytes, retention: str = "short", ttl: float | None = None) -> bool:
        return (await self._call(W.Set(key, value, retention, ttl_seconds=ttl))).ok

    async def batch_set(self, keys, values, retention: str = "short") -> list[bool]:
        return (await self._call(W.BatchSet(keys, values, retention))).ok

    async def set_lease(self, key: bytes, size: int, retention: str = "short") -> W.SetReserveResponse:
        return await self._call(W.SetReserve(key, size, retention))

    async def commit_set(self, lease: W.SetReserveResponse, data) -> bool:
        self.arena.write_payload(lease.payload_offset, data)
        return (await self._call(W.SetCommit(lease.lease_token, len(data)))).ok

    async def cancel_set(self, lease: W.SetReserveResponse) -> bool:
        return (await self._call(W.SetCancel(lease.lease_token))).ok

    async def exists(self, keys: list[bytes]) -> list[bool]:
        return (await self._call(W.Exists(keys))).present

    async def lookup_tier(self, key: bytes) -> W.LookupTierResponse:
        return await self._call(W.LookupTier(key))

    async def prefetch_hint(self, keys: list[bytes]) -> list[bool]:
        return (await self._call(W.PrefetchHint(keys))).present

    async def clear(self) -> int:
        return (await self._call(W.Clear())).cleared_entries

    async def stats(self) -> W.StatsResponse:
        return await self._call(W.Stats())

    async def close(self) -> None:
        if self.writer is not None:
            self.writer.close()
        if self.arena is not None:
            self.arena.close()


def hash_key(h: int) -> bytes:
    """8-byte key of a chained block hash."""
    return int(h).to_bytes(8, "little", signed=False)


class SyncKvdStore:
    """Blocking facade over :class:`KvdClient` (its own event-loop thread) with
    the ``set / get / exists`` surface the engine's tier manager uses."""

    def __init__(self, path: str, shared_arena: bool = True):
        import threading

        self.loop = asyncio.new_event_loop()
        self._t = threading.Thread(target=self.loop.run_forever, daemon=True)
        self._t.start()
        self.client = KvdClient(path, "infera-b200-engine")
        self._run(self.client.connect(shared_arena=shared_arena))

    def _run(self, coro):
        return asyncio.run_coroutine_threadsafe(coro, self.loop).result()

    def set(self, key: bytes, value, retention: str = "long") -> bool:
        return self._run(self.client.set(key, bytes(value), retention))

    def get(self, key: bytes) -> bytes | None:
        return self._run(self.client.get(key))

    def exists(self, key: bytes) -> bool:
        return self._run(self.client.exists([key]))[0]

    def register_arena(self):
        """Page-lock the shared arena for device copies; a uint8 tensor over
        it, or None (no arena / no GPU)."""
        if self.client.arena is None:
            return None
        if getattr(self, "_arena_t", None) is None:
            self._arena_t = self.client.arena.register_cuda()
        return self._arena_t

    def read_shared(self, key: bytes):
        """(arena view, payload offset, size, version) of an arena-held value,
        or None (then use :meth:`get`)."""
        if self.client.arena is None:
            return None
        r = self._run(self.client.get_shared(key))
        return None if r is None else (self.client.arena, *r)

    def exists_many(self, keys: list[bytes]) -> list[bool]:
        """One round trip for a run of keys (the tier manager's hit count)."""
        return self._run(self.client.exists(list(keys)))

    def close(self) -> None:
        self._run(self.client.close())
        self.loop.call_soon_threadsafe(self.loop.stop)


class KvdPrefetchClient:
    """Router side: one short-lived connection per prewarm request."""

    def __init__(self, path: str):
        self.path = path

    async def prefetch_hint(self, hashes: list[int], retention: str = "long") -> bool:
        try:
            c = KvdClient(self.path, "infera-b200-router")
            await c.connect()
            await c.prefetch_hint([hash_key(h) for h in hashes])
            await c.close()
            return True
        except (OSError, ConnectionError):
            return False

"""The KV tier daemon: asyncio Unix-socket server over the host store.

Per connection: HELLO (optionally negotiating the shared arena, whose memfd
is then sent with SCM_RIGHTS), then any mix of GET / BATCH_GET (inline bytes,
or arena offsets + versions for arena clients), SET / BATCH_SET,
SET_RESERVE -> client writes the leased arena slot in place -> SET_COMMIT /
SET_CANCEL (leases of a client that disconnects are cancelled), EXISTS,
LOOKUP_TIER, REGISTER_FILE_ENTRY, PREFETCH_HINT (a background worker
promotes L3 entries into RAM ahead of the request), CLEAR, STATS.
Behaviour of ``infera/kvd/server.py:76-1592``.

    python -m infera_b200.kvd --socket /tmp/kvd.sock --ram-gib 64 --slot-mib 4 --l3-dir /nvme/kvd
"""

from __future__ import annotations

import argparse
import asyncio
import itertools
import logging
import os

from infera_b200.kvd import wire as W
from infera_b200.kvd.fd_passing import async_send_fd
from infera_b200.kvd.shared_arena import SharedArena
from infera_b200.kvd.store import HostStore
from infera_b200.kvd.tablespace import Tablespace

logger = logging.getLogger(__name__)


class KvdServer:
    def __init__(self, socket_path: str, store: HostStore, server_id: str = "infera-b200-kvd"):
        self.path = socket_path
        self.store = store
        self.server_id = server_id
        self._leases: dict[int, tuple] = {}
        self._lease_ids = itertools.count(1)
        self._prefetch_q: asyncio.Queue | None = None
        self._server = None
        self._worker = None

    async def start(self) -> None:
        if os.path.exists(self.path):
            os.unlink(self.path)
        self._prefetch_q = asyncio.Queue()
        self._server = await asyncio.start_unix_server(self._client, path=self.path)
        self._worker = asyncio.create_task(self._prefetch_worker())

    async def stop(self) -> None:
        if self._worker:
            self._worker.cancel()
        if self._server:
            self._server.close()
            await self._server.wait_closed()
        if os.path.exists(self.path):
            os.unlink(self.path)

    async def _prefetch_worker(self) -> None:
        while True:
            key = await self._prefetch_q.get()
            await asyncio.get_running_loop().run_in_executor(None, self.store.get_entry, key)

    async def _client(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter) -> None:
        shared = False
        my_leases: set[int] = set()
        try:
            while True:
                try:
                    msg = await W.read_frame(reader)
                except (asyncio.IncompleteReadError, ConnectionError):
                    return
                except ValueError as e:
                    await W.write_frame(writer, W.ErrorMessage("bad_frame", str(e)))
                    continue
                if isinstance(msg, W.Hello):
                    arena = self.store.arena
                    if msg.prefers_shared_arena and arena is not None:
                        shared = True
                        await W.write_frame(writer, W.HelloAck(self.server_id, 1,
                                                               (arena.size, arena.slot_size, os.getpid())))
                        await async_send_fd(writer, arena.fd)
                    else:
                        await W.write_frame(writer, W.HelloAck(self.server_id, 1, None))
                    continue
                resp = self._dispatch(msg, shared, my_leases)
                await W.write_frame(writer, resp)
        finally:
            for tok in my_leases:
                lease = self._leases.pop(tok, None)
                if lease is not None:
                    self.store.cancel(lease[1], lease[2])
            writer.close()

    def _dispatch(self, msg, shared: bool, my_leases: set):
        st = self.store
        if isinstance(msg, W.Get):
            e = st.get_entry(msg.key)
            if e is None:
                return W.GetResponse(None)
            if shared and e.slot is not None:
                return W.GetSharedResponse(st.arena.payload_offset(e.slot), e.size, e.version, e.retention)
            return W.GetResponse(st._read(e), e.retention)
        if isinstance(msg, W.BatchGet):
            if shared and st.arena is not None:
                out = []
                for k in msg.keys:
                    e = st.get_entry(k)
                    out.append(None if e is None or e.slot is None else
                               (st.arena.payload_offset(e.slot), e.size, e.version))
                return W.BatchGetSharedResponse(out)
            return W.BatchGetResponse([st.get(k) for k in msg.keys])
        if isinstance(msg, W.Set):
            ok = st.set(msg.key, msg.value, msg.retention, msg.ttl_seconds)
            return W.SetAck(ok, "" if ok else "rejected: store full of higher-priority entries")
        if isinstance(msg, W.BatchSet):
            return W.BatchSetAck([st.set(k, v, msg.retention, msg.ttl_seconds) for k, v in zip(msg.keys, msg.values)])
        if isinstance(msg, W.SetReserve):
            r = st.reserve(msg.key, msg.size, msg.retention, msg.ttl_seconds)
            if r is None:
                return W.SetReserveResponse(False, reason="no arena slot available")
            slot, off = r
            tok = next(self._lease_ids)
            self._leases[tok] = (msg.key, slot, msg.size, msg.retention, msg.ttl_seconds)
            my_leases.add(tok)
            return W.SetReserveResponse(True, tok, slot, off, st.arena.payload_max)
        if isinstance(msg, W.SetCommit):
            lease = self._leases.pop(msg.lease_token, None)
            my_leases.discard(msg.lease_token)
            if lease is None:
                return W.SetCommitResponse(False, "unknown lease")
            key, slot, reserved, ret, ttl = lease
            st.commit(key, slot, msg.size, reserved, ret, ttl)
            return W.SetCommitResponse(True)
        if isinstance(msg, W.SetCancel):
            lease = self._leases.pop(msg.lease_token, None)
            my_leases.discard(msg.lease_token)
            if lease is not None:
                st.cancel(lease[1], lease[2])
            return W.SetCancelResponse(lease is not None)
        if isinstance(msg, W.Exists):
            return W.ExistsResponse([st.exists(k) for k in msg.keys])
        if isinstance(msg, W.LookupTier):
            tier = st.tier(msg.key)
            if tier == "file":
                if msg.key in st.file_entries:
                    path, off, size, ver, ret = st.file_entries[msg.key]
                    return W.LookupTierResponse("file", path, off, size, ver, ret)
                loc = st.l3.location(msg.key)
                if loc is not None:
                    path, off, size, ver = loc
                    return W.LookupTierResponse("file", path, off, size, ver, st.l3.index[msg.key].retention)
            if tier == "ram":
                e = st.entries[msg.key]
                return W.LookupTierResponse("ram", size=e.size, version=e.version, retention=e.retention)
            return W.LookupTierResponse("miss")
        if isinstance(msg, W.RegisterFileEntry):
            st.file_entries[msg.key] = (msg.path, msg.file_offset, msg.size, msg.version, msg.retention)
            return W.RegisterFileEntryAck(True)
        if isinstance(msg, W.PrefetchHint):
            for k in msg.keys:
                if st.tier(k) == "file":
                    self._prefetch_q.put_nowait(k)
            return W.ExistsResponse([st.exists(k) for k in msg.keys])
        if isinstance(msg, W.Clear):
            return W.ClearAck(st.clear())
        if isinstance(msg, W.Stats):
            l3 = st.l3.bytes_used() if st.l3 is not None else 0
            return W.StatsResponse(len(st.entries), st.used, 0, l3, st.stats["gets"], st.stats["sets"],
                                   st.stats["hits"], st.stats["misses"], st.stats["evictions"])
        return W.ErrorMessage("unsupported", type(msg).__name__)


def build_store(ram_bytes: int, slot_bytes: int, l3_dir: str | None, l3_container_bytes: int = 1 << 30) -> HostStore:
    arena = SharedArena(max(1, ram_bytes // slot_bytes), slot_bytes) if slot_bytes else None
    l3 = Tablespace(l3_dir, container_bytes=l3_container_bytes,
                    slot_bytes=min(1 << 16, l3_container_bytes)) if l3_dir else None
    return HostStore(ram_bytes, arena=arena, l3=l3)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="python -m infera_b200.kvd")
    ap.add_argument("--socket", default="/tmp/infera-kvd.sock")
    ap.add_argument("--ram-gib", type=float, default=8.0)
    ap.add_argument("--slot-mib", type=float, default=4.0)
    ap.add_argument("--l3-dir", default=None)
    ap.add_argument("--l3-container-gib", type=float, default=1.0)
    a = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO)
    store = build_store(int(a.ram_gib * (1 << 30)), int(a.slot_mib * (1 << 20)), a.l3_dir,
                        int(a.l3_container_gib * (1 << 30)))

    async def run():
        srv = KvdServer(a.socket, store)
        await srv.start()
        logger.info("kvd listening on %s", a.socket)
        await asyncio.Event().wait()

    asyncio.run(run())


if __name__ == "__main__":
    main()

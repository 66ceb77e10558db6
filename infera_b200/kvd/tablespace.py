"""L3 tier: a tablespace of fixed-size container files on local NVMe.

* Container files ``ts_NNNN.dat`` of ``container_bytes`` (default 1 GiB),
  each cut into ``slot_bytes`` slots (default 64 KiB). An entry occupies a
  contiguous run of slots inside one container (first fit over a bitset).
* Every PUT reserves slots, writes the payload (``pwrite`` + fsync), then
  appends a journal record (+ fsync); only then is the entry visible. A
  DELETE appends a journal record. A crash between the two leaves slots that
  no journal record owns - they are free again after restart.
* Restart = load ``index.snapshot`` (msgpack) + replay ``index.log``;
  ``checkpoint()`` writes a new snapshot atomically and truncates the log.
* Where the filesystem allows it, payload I/O uses O_DIRECT with 4 KiB
  aligned buffers; otherwise buffered I/O.

Design of ``infera/kvd/tablespace.py:204-1805`` (container / slot /
journal / snapshot), written for this daemon.
"""

from __future__ import annotations

import mmap
import os
import struct
import threading
import time
import zlib
from dataclasses import dataclass

import msgpack

ALIGN = 4096
_REC = struct.Struct("<II")  # length, crc32


@dataclass
class Extent:
    container: int
    slot: int
    nslots: int
    size: int
    retention: str
    version: int
    created: float


class _Bitset:
    def __init__(self, n: int):
        self.n = n
        self.bits = bytearray(n)

    def find_run(self, k: int) -> int | None:
        run = 0
        for i in range(self.n):
            if self.bits[i]:
                run = 0
            else:
                run += 1
                if run == k:
                    return i - k + 1
        return None

    def set(self, start: int, k: int, v: int) -> None:
        for i in range(start, start + k):
            self.bits[i] = v

    def used(self) -> int:
        return sum(self.bits)


def _aligned_buffer(n: int) -> mmap.mmap:
    return mmap.mmap(-1, max(ALIGN, (n + ALIGN - 1) // ALIGN * ALIGN))


class Tablespace:
    def __init__(self, root: str, *, container_bytes: int = 1 << 30, slot_bytes: int = 1 << 16,
                 max_containers: int = 64, fsync: bool = True, direct_io: bool | None = None):
        if container_bytes % slot_bytes or slot_bytes % ALIGN:
            raise ValueError("container size must be a multiple of the slot size, slots 4 KiB aligned")
        self.root = root
        self.container_bytes = container_bytes
        self.slot_bytes = slot_bytes
        self.slots_per_container = container_bytes // slot_bytes
        self.max_containers = max_containers
        self.fsync = fsync
        os.makedirs(root, exist_ok=True)
        self.index: dict[bytes, Extent] = {}
        self.bitsets: list[_Bitset] = []
        self.fds: list[int] = []
        self.lock = threading.RLock()
        self.direct = self._probe_direct() if direct_io is None else direct_io
        self.version = 0
        self.stats = {"puts": 0, "gets": 0, "deletes": 0, "bytes_written": 0, "bytes_read": 0}
        self._restore()
        self.journal = open(os.path.join(root, "index.log"), "ab")

    # ------------------------------------------------------------------ files
    def _probe_direct(self) -> bool:
        path = os.path.join(self.root, ".odirect_probe")
        try:
            fd = os.open(path, os.O_RDWR | os.O_CREAT | getattr(os, "O_DIRECT", 0), 0o644)
            buf = _aligned_buffer(ALIGN)
            os.pwrite(fd, buf, 0)
            os.close(fd)
            os.unlink(path)
            return hasattr(os, "O_DIRECT")
        except OSError:
            try:
                os.unlink(path)
            except OSError:
                pass
            return False

    def _container_path(self, i: int) -> str:
        return os.path.join(self.root, f"ts_{i:04d}.dat")

    def _open_container(self, i: int) -> None:
        while len(self.fds) <= i:
            j = len(self.fds)
            flags = os.O_RDWR | os.O_CREAT | (getattr(os, "O_DIRECT", 0) if self.direct else 0)
            fd = os.open(self._container_path(j), flags, 0o644)
            if os.fstat(fd).st_size < self.container_bytes:
                os.ftruncate(fd, self.container_bytes)
            self.fds.append(fd)
            self.bitsets.append(_Bitset(self.slots_per_container))

    # ------------------------------------------------------------------ journal
    def _journal_append(self, rec: dict) -> None:
        body = msgpack.packb(rec, use_bin_type=True)
        self.journal.write(_REC.pack(len(body), zlib.crc32(body)) + body)
        self.journal.flush()
        if self.fsync:
            os.fsync(self.journal.fileno())

    @staticmethod
    def _read_records(path: str):
        try:
            data = open(path, "rb").read()
        except FileNotFoundError:
            return
        off = 0
        while off + _REC.size <= len(data):
            n, crc = _REC.unpack_from(data, off)
            body = data[off + _REC.size: off + _REC.size + n]
            if len(body) < n or zlib.crc32(body) != crc:
                return  # torn tail from a crash: stop replay here
            yield msgpack.unpackb(body, raw=False)
            off += _REC.size + n

    def _apply(self, rec: dict) -> None:
        if rec["t"] == "put":
            e = Extent(rec["c"], rec["s"], rec["n"], rec["size"], rec["r"], rec["v"], rec["ts"])
            old = self.index.get(rec["k"])
            if old is not None:
                self.bitsets[old.container].set(old.slot, old.nslots, 0)
            self._open_container(e.container)
            self.bitsets[e.container].set(e.slot, e.nslots, 1)
            self.index[rec["k"]] = e
            self.version = max(self.version, e.version)
        elif rec["t"] == "del":
            e = self.index.pop(rec["k"], None)
            if e is not None:
                self.bitsets[e.container].set(e.slot, e.nslots, 0)

    def _restore(self) -> None:
        snap = os.path.join(self.root, "index.snapshot")
        if os.path.exists(snap):
            with open(snap, "rb") as f:
                data = msgpack.unpackb(f.read(), raw=False)
            for k, e in data["entries"]:
                self._apply({"t": "put", "k": k, "c": e[0], "s": e[1], "n": e[2], "size": e[3], "r": e[4],
                             "v": e[5], "ts": e[6]})
        for rec in self._read_records(os.path.join(self.root, "index.log")):
            self._apply(rec)

    def checkpoint(self) -> None:
        """Atomic snapshot of the index, then an empty journal."""
        with self.lock:
            entries = [(k, [e.container, e.slot, e.nslots, e.size, e.retention, e.version, e.created])
                       for k, e in self.index.items()]
            tmp = os.path.join(self.root, "index.snapshot.tmp")
            with open(tmp, "wb") as f:
                f.write(msgpack.packb({"entries": entries}, use_bin_type=True))
                f.flush()
                os.fsync(f.fileno())
            os.replace(tmp, os.path.join(self.root, "index.snapshot"))
            self.journal.close()
            self.journal = open(os.path.join(self.root, "index.log"), "wb")

    # ------------------------------------------------------------------ data
    def _reserve(self, nslots: int) -> tuple[int, int] | None:
        for c in range(self.max_containers):
            self._open_container(c)
            s = self.bitsets[c].find_run(nslots)
            if s is not None:
                self.bitsets[c].set(s, nslots, 1)
                return c, s
        return None

    def put(self, key: bytes, value, retention: str = "short") -> bool:
        n = len(value)
        nslots = max(1, (n + self.slot_bytes - 1) // self.slot_bytes)
        if nslots > self.slots_per_container:
            return False
        with self.lock:
            where = self._reserve(nslots)
            if where is None:
                return False
            c, s = where
            buf = _aligned_buffer(n)
            buf[:n] = value
            os.pwrite(self.fds[c], memoryview(buf)[: (n + ALIGN - 1) // ALIGN * ALIGN], s * self.slot_bytes)
            if self.fsync:
                os.fsync(self.fds[c])
            self.version += 1
            rec = {"t": "put", "k": key, "c": c, "s": s, "n": nslots, "size": n, "r": retention, "v": self.version,
                   "ts": time.time()}
            old = self.index.get(key)
            self._journal_append(rec)
            if old is not None:
                self.bitsets[old.container].set(old.slot, old.nslots, 0)
            self.index[key] = Extent(c, s, nslots, n, retention, self.version, rec["ts"])
            self.stats["puts"] += 1
            self.stats["bytes_written"] += n
            return True

    def get(self, key: bytes) -> bytes | None:
        with self.lock:
            e = self.index.get(key)
            if e is None:
                return None
            buf = _aligned_buffer(e.size)
            nread = (e.size + ALIGN - 1) // ALIGN * ALIGN
            os.preadv(self.fds[e.container], [memoryview(buf)[:nread]], e.slot * self.slot_bytes)
            self.stats["gets"] += 1
            self.stats["bytes_read"] += e.size
            return bytes(buf[: e.size])

    def location(self, key: bytes) -> tuple[str, int, int, int] | None:
        e = self.index.get(key)
        if e is None:
            return None
        return self._container_path(e.container), e.slot * self.slot_bytes, e.size, e.version

    def delete(self, key: bytes) -> bool:
        with self.lock:
            if key not in self.index:
                return False
            self._journal_append({"t": "del", "k": key})
            e = self.index.pop(key)
            self.bitsets[e.container].set(e.slot, e.nslots, 0)
            self.stats["deletes"] += 1
            return True

    def __contains__(self, key: bytes) -> bool:
        return key in self.index

    def __len__(self) -> int:
        return len(self.index)

    def bytes_used(self) -> int:
        return sum(e.size for e in self.index.values())

    def evict_lru(self, need_bytes: int, priority) -> int:
        """Drop oldest lowest-priority entries until ``need_bytes`` are freed."""
        freed = 0
        with self.lock:
            order = sorted(self.index.items(), key=lambda kv: (priority(kv[1].retention), kv[1].created))
            for k, e in order:
                if freed >= need_bytes:
                    break
                self.delete(k)
                freed += e.nslots * self.slot_bytes
        return freed

    def close(self) -> None:
        with self.lock:
            self.journal.close()
            for fd in self.fds:
                os.close(fd)
            self.fds = []

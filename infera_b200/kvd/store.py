"""L2 host store: priority-aware LRU over the shared arena (or plain bytes).

* Retention priorities: none 0 < ephemeral 10 < short 50 < long 100.
  Eviction takes the least recently used entry of the LOWEST priority; a
  write that could only be admitted by displacing a higher-priority entry is
  rejected instead.
* Evicted entries spill to the L3 tablespace when one is configured; a GET
  that misses RAM but hits L3 promotes the entry back into RAM.
* ``ttl_seconds`` expires an entry lazily on access.

Behaviour of ``infera/kvd/store.py:84-1241``.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from dataclasses import dataclass

from infera_b200.kvd.wire import RETENTION_PRIORITY


@dataclass
class Entry:
    size: int
    retention: str
    slot: int | None = None        # arena slot, or None when stored inline
    value: bytes | None = None
    version: int = 0
    expires: float | None = None


class HostStore:
    def __init__(self, capacity_bytes: int, arena=None, l3=None):
        self.capacity = capacity_bytes if arena is None else arena.num_slots * arena.payload_max
        self.arena = arena
        self.l3 = l3
        self.entries: dict[bytes, Entry] = {}
        self.lru: dict[int, OrderedDict] = {p: OrderedDict() for p in sorted(set(RETENTION_PRIORITY.values()))}
        self.used = 0
        self.lock = threading.RLock()
        self.file_entries: dict[bytes, tuple] = {}
        self.stats = {"gets": 0, "sets": 0, "hits": 0, "misses": 0, "evictions": 0, "spills": 0, "promotions": 0,
                      "rejected": 0}
        # fn(key, spilled: bool): an entry left host memory (to the NVMe tier
        # when spilled); the engine's tier manager reports it to the KV index
        self.listeners: list = []

    def add_listener(self, fn) -> None:
        self.listeners.append(fn)

    @staticmethod
    def _prio(retention: str) -> int:
        return RETENTION_PRIORITY.get(retention, RETENTION_PRIORITY["short"])

    def _touch(self, key: bytes, e: Entry) -> None:
        q = self.lru[self._prio(e.retention)]
        q.pop(key, None)
        q[key] = None

    def _drop(self, key: bytes, spill: bool) -> None:
        e = self.entries.pop(key)
        self.lru[self._prio(e.retention)].pop(key, None)
        self.used -= e.size
        spilled = False
        if spill and self.l3 is not None:
            data = self._read(e)
            if data is not None and self.l3.put(key, data, e.retention):
                self.stats["spills"] += 1
                spilled = True
        if e.slot is not None:
            self.arena.free(e.slot)
        for fn in self.listeners:
            try:
                fn(key, spilled)
            except Exception:
                pass

    def _read(self, e: Entry) -> bytes | None:
        if e.slot is None:
            return e.value
        off = self.arena.payload_offset(e.slot)
        return bytes(self.arena.view[off: off + e.size])

    def _make_room(self, size: int, prio: int) -> bool:
        need_slot = self.arena is not None
        while self.used + size > self.capacity or (need_slot and self.arena.free_slots() == 0):
            victim = None
            for p, q in self.lru.items():
                if q and p <= prio:
                    victim = next(iter(q))
                    break
            if victim is None:
                return False
            self._drop(victim, spill=True)
            self.stats["evictions"] += 1
        return True

    # ------------------------------------------------------------------ API
    def set(self, key: bytes, value, retention: str = "short", ttl: float | None = None) -> bool:
        size = len(value)
        if self.arena is not None and size > self.arena.payload_max:
            return False
        with self.lock:
            self.stats["sets"] += 1
            if key in self.entries:
                self._drop(key, spill=False)
            if not self._make_room(size, self._prio(retention)):
                self.stats["rejected"] += 1
                return False
            e = Entry(size, retention, expires=(time.monotonic() + ttl) if ttl else None)
            if self.arena is not None:
                e.slot = self.arena.alloc()
                e.version = self.arena.write(e.slot, value)
            else:
                # a buffer built for this call (a packed chunk) is kept as is
                e.value = value if isinstance(value, (bytes, bytearray)) else bytes(value)
            self.entries[key] = e
            self.used += size
            self._touch(key, e)
            return True

    def reserve(self, key: bytes, size: int, retention: str = "short", ttl: float | None = None):
        """Lease an arena slot for an in-place write; returns (slot, offset)."""
        if self.arena is None or size > self.arena.payload_max:
            return None
        with self.lock:
            if key in self.entries:
                self._drop(key, spill=False)
            if not self._make_room(size, self._prio(retention)):
                self.stats["rejected"] += 1
                return None
            slot = self.arena.alloc()
            self.arena.begin_write(slot)
            self.used += size
            return slot, self.arena.payload_offset(slot)

    def commit(self, key: bytes, slot: int, size: int, reserved: int, retention: str, ttl: float | None) -> None:
        with self.lock:
            e = Entry(size, retention, slot=slot, expires=(time.monotonic() + ttl) if ttl else None)
            e.version = self.arena.end_write(slot, size)
            self.used += size - reserved
            self.entries[key] = e
            self._touch(key, e)
            self.stats["sets"] += 1

    def cancel(self, slot: int, reserved: int) -> None:
        with self.lock:
            self.arena.end_write(slot, 0)
            self.arena.free(slot)
            self.used -= reserved

    def _live(self, key: bytes) -> Entry | None:
        e = self.entries.get(key)
        if e is not None and e.expires is not None and time.monotonic() > e.expires:
            self._drop(key, spill=False)
            return None
        return e

    def get_entry(self, key: bytes, promote: bool = True) -> Entry | None:
        with self.lock:
            self.stats["gets"] += 1
            e = self._live(key)
            if e is None and promote and self.l3 is not None and key in self.l3:
                data = self.l3.get(key)
                ext = self.l3.index.get(key)
                if data is not None and self.set(key, data, ext.retention if ext else "short"):
                    self.stats["promotions"] += 1
                    self.stats["sets"] -= 1
                    e = self.entries.get(key)
            if e is None:
                self.stats["misses"] += 1
                return None
            self.stats["hits"] += 1
            self._touch(key, e)
            return e

    def get(self, key: bytes) -> bytes | None:
        e = self.get_entry(key)
        return None if e is None else self._read(e)

    def read(self, key: bytes) -> bytes | None:
        """The value from host memory, or straight from the NVMe tier
        without promoting it into host memory (a reader that copies it
        onward - the engine promoting into HBM - needs no host copy kept)."""
        with self.lock:
            self.stats["gets"] += 1
            e = self._live(key)
            if e is not None:
                self.stats["hits"] += 1
                self._touch(key, e)
                return self._read(e)
            data = self.l3.get(key) if self.l3 is not None and key in self.l3 else None
            self.stats["hits" if data is not None else "misses"] += 1
            return data

    def exists_many(self, keys: list[bytes]) -> list[bool]:
        return [self.exists(k) for k in keys]

    def exists(self, key: bytes) -> bool:
        with self.lock:
            return self._live(key) is not None or (self.l3 is not None and key in self.l3) or key in self.file_entries

    def tier(self, key: bytes) -> str:
        with self.lock:
            if self._live(key) is not None:
                return "ram"
            if (self.l3 is not None and key in self.l3) or key in self.file_entries:
                return "file"
            return "miss"

    def clear(self) -> int:
        with self.lock:
            n = len(self.entries)
            for k in list(self.entries):
                self._drop(k, spill=False)
            return n

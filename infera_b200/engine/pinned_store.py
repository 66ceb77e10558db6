"""In-process host KV tier held in one page-locked arena: page slots that
the device reads and writes by DMA, with no per-page host-side copies.

The arena is a pinned host tensor [slots, page elements] (one page of every
layer's K and V, page-major: the layout of one v2 chunk payload). The
engine's tier manager gathers evicted pages on the device into its staging
ring and copies each staging slot straight into the slot this store
reserved for the block; a promote copies the slot straight back into the
device staging buffer. So a save or a promote costs one DMA per page at the
host link's rate, against a pack + copy in Python per page for a store of
byte blobs.

Slots are kept in LRU order. A slot is reserved (being written: not visible
to lookups), then committed once its copy has landed. A slot being read by
a promote is pinned and never reused until released. Dropping a committed
block (LRU eviction to make room) notifies the listeners the same way the
byte-blob host store does (``listener(key, spilled)``), so the tier-aware
KV index follows.

The reference keeps its host tier in the kvd daemon's shared arena
(``infera/kvd/shared_arena.py``, ``infera/kvd/store.py``); this is the
single-process form of the same idea for the engine's own tier.
"""

from __future__ import annotations

import threading
from collections import OrderedDict

import torch


class PinnedPageStore:
    def __init__(self, capacity_bytes: int, page_bytes: int = 0):
        self.capacity_bytes = int(capacity_bytes)
        self.page_bytes = int(page_bytes)
        self.arena: torch.Tensor | None = None     # [slots, page elements], sized by bind()
        self.n_slots = 0
        self._lock = threading.Lock()
        self._slot_of: dict[bytes, int] = {}
        self._lru: OrderedDict[bytes, None] = OrderedDict()   # committed keys, oldest first
        self._pending: dict[bytes, int] = {}                  # reserved, copy in flight
        self._pins: dict[int, int] = {}                       # slot -> readers
        self._free: list[int] = []
        self.listeners = []
        self.stats = {"stored": 0, "evicted": 0, "reserve_failed": 0}

    # ------------------------------------------------------------------ setup
    def bind(self, page_elems: int, dtype: torch.dtype, pin: bool = True) -> torch.Tensor:
        """Allocate the arena for pages of ``page_elems`` elements (called by
        the tier manager, which knows the cache geometry)."""
        if self.arena is not None:
            return self.arena
        esize = torch.empty(0, dtype=dtype).element_size()
        self.page_bytes = page_elems * esize
        self.n_slots = max(1, self.capacity_bytes // self.page_bytes)
        self.arena = torch.empty(self.n_slots, page_elems, dtype=dtype, pin_memory=pin)
        self._free = list(range(self.n_slots - 1, -1, -1))
        return self.arena

    def add_listener(self, fn) -> None:
        self.listeners.append(fn)

    # ------------------------------------------------------------------ lookups
    def exists(self, key: bytes) -> bool:
        with self._lock:
            return key in self._lru

    def exists_many(self, keys: list[bytes]) -> list[bool]:
        with self._lock:
            return [k in self._lru for k in keys]

    def __len__(self) -> int:
        with self._lock:
            return len(self._lru)

    # ------------------------------------------------------------------ writes
    def _take_slot(self, dropped: list[bytes]) -> int | None:
        if self._free:
            return self._free.pop()
        for key in self._lru:                 # oldest first, skipping slots a promote is reading
            slot = self._slot_of[key]
            if self._pins.get(slot, 0) == 0:
                del self._lru[key]
                del self._slot_of[key]
                dropped.append(key)
                self.stats["evicted"] += 1
                return slot
        return None

    def reserve(self, keys: list[bytes]) -> list[int | None]:
        """A slot for each key to be written: None when the key is already
        held or being written, -1 when no slot can be freed. Reserved slots
        stay invisible until :meth:`commit`."""
        out, dropped = [], []
        with self._lock:
            for key in keys:
                if key in self._lru or key in self._pending:
                    out.append(None)
                    continue
                slot = self._take_slot(dropped)
                if slot is None:
                    self.stats["reserve_failed"] += 1
                    out.append(-1)
                    continue
                self._pending[key] = slot
                out.append(slot)
        self._notify(dropped)
        return out

    def commit(self, keys: list[bytes]) -> list[bytes]:
        """The copies into these keys' reserved slots have landed."""
        done = []
        with self._lock:
            for key in keys:
                slot = self._pending.pop(key, None)
                if slot is None:
                    continue
                self._slot_of[key] = slot
                self._lru[key] = None
                self.stats["stored"] += 1
                done.append(key)
        return done

    def abort(self, keys: list[bytes]) -> None:
        with self._lock:
            for key in keys:
                slot = self._pending.pop(key, None)
                if slot is not None:
                    self._free.append(slot)

    # ------------------------------------------------------------------ reads
    def acquire(self, keys: list[bytes]) -> list[int]:
        """Slots of the leading run of committed keys, pinned against reuse
        (and refreshed in LRU order) until :meth:`release`."""
        out = []
        with self._lock:
            for key in keys:
                if key not in self._lru:
                    break
                slot = self._slot_of[key]
                self._lru.move_to_end(key)
                self._pins[slot] = self._pins.get(slot, 0) + 1
                out.append(slot)
        return out

    def release(self, slots: list[int]) -> None:
        with self._lock:
            for slot in slots:
                n = self._pins.get(slot, 0) - 1
                if n <= 0:
                    self._pins.pop(slot, None)
                else:
                    self._pins[slot] = n

    def delete(self, key: bytes) -> bool:
        with self._lock:
            if key not in self._lru:
                return False
            slot = self._slot_of[key]
            if self._pins.get(slot, 0):
                return False
            del self._lru[key]
            del self._slot_of[key]
            self._free.append(slot)
        self._notify([key])
        return True

    def _notify(self, keys: list[bytes]) -> None:
        for key in keys:
            for fn in self.listeners:
                try:
                    fn(key, False)
                except Exception:
                    pass

"""Budgeted eviction of file-per-chunk L3 caches.

A KV connector that stores one file per chunk (``<digest>.<retention>.kvcache``
in a directory) needs the directory kept under a byte budget
(``INFERA_KVD_L3_BUDGET_BYTES``) and the filesystem above a free-space
floor. The reaper scans the directory, and evicts by retention priority
(none < ephemeral < short < long) then least-recently-used (file atime /
mtime), until both limits hold. ``startup_budget_clamp`` shrinks a budget
that the disk cannot actually hold; ``write_with_reap`` retries a write
once after reaping when the disk is full (ENOSPC). Behaviour of
``infera/engine/vllm/_l3_reaper.py:64-405``.
"""

from __future__ import annotations

import errno
import os
import shutil
import threading
from dataclasses import dataclass

SUFFIX = ".kvcache"
PRIORITY = {"none": 0, "ephemeral": 10, "short": 50, "long": 100}


@dataclass
class CacheFile:
    path: str
    size: int
    retention: str
    last_use: float


def retention_of(name: str) -> str:
    parts = name[: -len(SUFFIX)].rsplit(".", 1) if name.endswith(SUFFIX) else [name]
    return parts[1] if len(parts) == 2 and parts[1] in PRIORITY else "short"


class L3FileReaper:
    def __init__(self, directory: str, budget_bytes: int | None = None, free_floor_bytes: int = 0,
                 disk_usage=shutil.disk_usage):
        self.dir = directory
        env = os.environ.get("INFERA_KVD_L3_BUDGET_BYTES")
        self.budget = budget_bytes if budget_bytes is not None else (int(env) if env else None)
        self.floor = free_floor_bytes
        self.disk_usage = disk_usage
        self.lock = threading.Lock()
        self.stats = {"scans": 0, "reaped_files": 0, "reaped_bytes": 0, "enospc_retries": 0}

    def scan(self) -> list[CacheFile]:
        out = []
        try:
            names = os.listdir(self.dir)
        except FileNotFoundError:
            return out
        for n in names:
            if not n.endswith(SUFFIX):
                continue
            p = os.path.join(self.dir, n)
            try:
                st = os.stat(p)
            except FileNotFoundError:
                continue
            out.append(CacheFile(p, st.st_size, retention_of(n), max(st.st_atime, st.st_mtime)))
        self.stats["scans"] += 1
        return out

    def startup_budget_clamp(self) -> int | None:
        """Clamp the budget to what the filesystem can hold above the floor."""
        if self.budget is None:
            return None
        du = self.disk_usage(self.dir)
        used = sum(f.size for f in self.scan())
        cap = max(0, used + du.free - self.floor)
        self.budget = min(self.budget, cap)
        return self.budget

    def reap(self, need_bytes: int = 0) -> int:
        """Evict until the budget and the free floor hold with ``need_bytes``
        more to write. Returns the bytes freed."""
        with self.lock:
            files = sorted(self.scan(), key=lambda f: (PRIORITY.get(f.retention, 50), f.last_use))
            used = sum(f.size for f in files)
            free = self.disk_usage(self.dir).free
            freed = 0
            for f in files:
                over_budget = self.budget is not None and used - freed + need_bytes > self.budget
                under_floor = free + freed - need_bytes < self.floor
                if not over_budget and not under_floor:
                    break
                try:
                    os.unlink(f.path)
                except FileNotFoundError:
                    continue
                freed += f.size
                self.stats["reaped_files"] += 1
                self.stats["reaped_bytes"] += f.size
            return freed

    def write_with_reap(self, name: str, data: bytes) -> str:
        path = os.path.join(self.dir, name)
        self.reap(len(data))
        for attempt in range(2):
            try:
                with open(path + ".tmp", "wb") as f:
                    f.write(data)
                os.replace(path + ".tmp", path)
                return path
            except OSError as e:
                if e.errno != errno.ENOSPC or attempt == 1:
                    raise
                self.stats["enospc_retries"] += 1
                self.reap(2 * len(data))
        return path


class _Ext:
    def __init__(self, retention: str):
        self.retention = retention


class FileChunkStore:
    """File-per-chunk NVMe tier (``<key hex>.<retention>.kvcache`` in one
    directory) with the reaper keeping it under its byte budget and above the
    free-space floor. It offers the L3 surface the host store spills to and
    promotes from (``put`` / ``get`` / ``in`` / ``index``), so the engine's
    tier can use it in place of the tablespace: ``kv_tier="host:<GiB>:files:
    <dir>"``. A file removed by the reaper simply misses on the next lookup.
    Role of the reference's file-per-chunk L3 of its vLLM connector with
    ``infera/engine/vllm/_l3_reaper.py``."""

    def __init__(self, directory: str, budget_bytes: int | None = None, free_floor_bytes: int = 0):
        os.makedirs(directory, exist_ok=True)
        self.dir = directory
        self.reaper = L3FileReaper(directory, budget_bytes, free_floor_bytes)
        self.reaper.startup_budget_clamp()
        self.index: dict[bytes, _Ext] = {}
        for f in self.reaper.scan():      # chunks left by an earlier run stay usable
            name = os.path.basename(f.path)
            try:
                key = bytes.fromhex(name.split(".", 1)[0])
            except ValueError:
                continue
            self.index[key] = _Ext(f.retention)

    def _name(self, key: bytes, retention: str) -> str:
        return f"{key.hex()}.{retention if retention in PRIORITY else 'short'}{SUFFIX}"

    def put(self, key: bytes, value, retention: str = "short") -> bool:
        try:
            self.reaper.write_with_reap(self._name(key, retention), bytes(value))
        except OSError:
            return False
        self.index[key] = _Ext(retention)
        return True

    def get(self, key: bytes) -> bytes | None:
        ext = self.index.get(key)
        if ext is None:
            return None
        path = os.path.join(self.dir, self._name(key, ext.retention))
        try:
            with open(path, "rb") as f:
                data = f.read()
            os.utime(path)            # recency for the reaper's LRU
            return data
        except FileNotFoundError:     # reaped
            self.index.pop(key, None)
            return None

    def __contains__(self, key: bytes) -> bool:
        ext = self.index.get(key)
        if ext is None:
            return False
        if not os.path.exists(os.path.join(self.dir, self._name(key, ext.retention))):
            self.index.pop(key, None)
            return False
        return True

    def delete(self, key: bytes) -> bool:
        ext = self.index.pop(key, None)
        if ext is None:
            return False
        try:
            os.unlink(os.path.join(self.dir, self._name(key, ext.retention)))
        except FileNotFoundError:
            pass
        return True

    def __len__(self) -> int:
        return len(self.index)

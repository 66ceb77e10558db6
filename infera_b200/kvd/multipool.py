"""Size-classed and striped L3 regions over :class:`Tablespace`.

* :class:`MultiPoolTablespace` - several tablespaces with different slot
  sizes (e.g. 64 KiB / 1 MiB / 16 MiB) under one root. A value goes to the
  pool whose slot size wastes least (the smallest slot size with at most
  ``max_slots`` slots for it), so small MLA chunks and large GQA chunks
  both pack densely. Keys are looked up in the pool that holds them.
* :class:`StripedTablespace` - one tablespace per device path (several
  NVMe drives); keys are sharded by hash, each shard has its own I/O worker
  so batched reads and writes run on all devices in parallel.

Roles of ``infera/kvd/tablespace_multipool.py:102`` and
``infera/kvd/striped_long_region.py:129``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import zlib

from infera_b200.kvd.tablespace import Tablespace


class MultiPoolTablespace:
    def __init__(self, root: str, slot_sizes=(1 << 16, 1 << 20, 1 << 24), container_bytes: int = 1 << 30,
                 max_containers_per_pool: int = 16, max_slots: int = 16, fsync: bool = True,
                 direct_io: bool | None = None):
        self.slot_sizes = sorted(slot_sizes)
        self.max_slots = max_slots
        self.pools = []
        for s in self.slot_sizes:
            cb = max(container_bytes // s * s, s * max_slots)
            self.pools.append(Tablespace(os.path.join(root, f"pool_{s >> 10}k"), container_bytes=cb, slot_bytes=s,
                                         max_containers=max_containers_per_pool, fsync=fsync, direct_io=direct_io))

    def pool_for(self, size: int) -> int:
        for i, s in enumerate(self.slot_sizes):
            if (size + s - 1) // s <= self.max_slots:
                return i
        return len(self.slot_sizes) - 1

    def _holder(self, key: bytes):
        for p in self.pools:
            if key in p:
                return p
        return None

    def put(self, key: bytes, value, retention: str = "short") -> bool:
        old = self._holder(key)
        target = self.pools[self.pool_for(len(value))]
        ok = target.put(key, value, retention)
        if ok and old is not None and old is not target:
            old.delete(key)
        return ok

    def get(self, key: bytes) -> bytes | None:
        p = self._holder(key)
        return None if p is None else p.get(key)

    def delete(self, key: bytes) -> bool:
        p = self._holder(key)
        return False if p is None else p.delete(key)

    def __contains__(self, key: bytes) -> bool:
        return self._holder(key) is not None

    def __len__(self) -> int:
        return sum(len(p) for p in self.pools)

    def bytes_used(self) -> int:
        return sum(p.bytes_used() for p in self.pools)

    def stats(self) -> dict:
        return {f"pool_{s >> 10}k": {"entries": len(p), "bytes": p.bytes_used()}
                for s, p in zip(self.slot_sizes, self.pools)}

    def close(self) -> None:
        for p in self.pools:
            p.close()


class StripedTablespace:
    def __init__(self, roots: list[str], **kw):
        if not roots:
            raise ValueError("no device paths")
        self.shards = [Tablespace(r, **kw) for r in roots]
        self.workers = [cf.ThreadPoolExecutor(max_workers=1, thread_name_prefix=f"l3-shard{i}")
                        for i in range(len(roots))]

    def shard_of(self, key: bytes) -> int:
        return zlib.crc32(key) % len(self.shards)

    def put(self, key: bytes, value, retention: str = "short") -> bool:
        i = self.shard_of(key)
        return self.workers[i].submit(self.shards[i].put, key, value, retention).result()

    def get(self, key: bytes) -> bytes | None:
        i = self.shard_of(key)
        return self.workers[i].submit(self.shards[i].get, key).result()

    def get_many(self, keys: list[bytes]) -> list[bytes | None]:
        futs = [self.workers[self.shard_of(k)].submit(self.shards[self.shard_of(k)].get, k) for k in keys]
        return [f.result() for f in futs]

    def put_many(self, items: list[tuple[bytes, bytes]], retention: str = "short") -> list[bool]:
        futs = [self.workers[self.shard_of(k)].submit(self.shards[self.shard_of(k)].put, k, v, retention)
                for k, v in items]
        return [f.result() for f in futs]

    def delete(self, key: bytes) -> bool:
        i = self.shard_of(key)
        return self.workers[i].submit(self.shards[i].delete, key).result()

    def __contains__(self, key: bytes) -> bool:
        return key in self.shards[self.shard_of(key)]

    def __len__(self) -> int:
        return sum(len(s) for s in self.shards)

    def close(self) -> None:
        for w in self.workers:
            w.shutdown(wait=True)
        for s in self.shards:
            s.close()

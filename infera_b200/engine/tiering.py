"""KV-cache tiering for the engine: HBM pages <-> host DRAM <-> NVMe.

* Save on eviction: pages the block manager evicts while scheduling a step
  (they held full, hashed prefix blocks) are queued; right after the
  schedule, before the forward pass can overwrite them, ONE gather kernel
  copies all of them (every layer's K and V, or a latent MLA cache's one
  row per token) into slots of a device staging ring on the compute stream,
  and ONE device-to-host copy on a side stream moves them to the matching
  pinned host slots. A writer thread packs each slot as a v2 KV chunk
  straight from pinned memory and stores it under the block's chained
  hash; the host store spills its own evictions to the NVMe tablespace.
  Nothing waits on the host: a full ring drops saves (counted), it never
  stalls a step.
* Promote on a prefix hit: the scheduler learns, at admission, how many
  blocks after the HBM prefix hit a tier holds (the external hit count),
  allocates pages for them and parks the request. A loader thread reads
  the blobs into a pinned double buffer (chunks of ``load_chunk`` pages),
  and per chunk issues one host-to-device copy and one scatter kernel on
  the side stream; the side stream first waits for the compute stream's
  work at the time of the request (so the pages' previous content has been
  saved). The engine polls the load's completion event each step and only
  then registers the pages in the prefix cache and lets the request run:
  the step loop never blocks on a promote. With ``async_load=False``
  (tensor-parallel ranks, which must make the same scheduling decisions in
  lockstep) the same chunked copies run inline on the compute stream.
* With a :class:`~infera_b200.engine.pinned_store.PinnedPageStore` (spec
  ``pinned:<GiB>``) the host tier is one page-locked arena of page slots:
  a save copies each staging slot straight into the slot reserved for its
  block (committed once the copy landed) and a promote copies the slot
  straight into device staging, so no page passes through Python.
* Every block the tiers gain or lose is reported through ``index_sink``
  (the engine's tier-aware KV index feed).

Keys are the 8-byte little-endian chained block hash, so any instance that
computed the same prefix produces the same keys. Role of the reference's
kvd connector for vLLM (``infera/engine/vllm/kvd_connector.py``: save on
eviction, ``get_num_new_matched_tokens`` at :1727, side-stream loads at
:2824 / :5824).
"""

from __future__ import annotations

import queue
import threading
import time

import numpy as np
import torch

from infera_b200.engine.packed_format import ChunkHeader, PackedFormatError, pack_chunk, unpack_chunk
from infera_b200.engine.pinned_store import PinnedPageStore
from infera_b200.kv.types import Tier
from infera_b200.ops import kernels as K


def hash_key(h: int) -> bytes:
    return int(h).to_bytes(8, "little", signed=False)


class TierManager:
    def __init__(self, k_cache: torch.Tensor, v_cache: torch.Tensor, store, page_size: int = 16,
                 retention: str = "long", staging_pages: int = 0, load_chunk: int = 32,
                 async_load: bool = True, key_tag: bytes = b""):
        self.k = k_cache
        self.v = v_cache
        self.store = store
        self.key_tag = key_tag      # appended to every key (a tensor-parallel rank's shard)
        self.ps = page_size
        self.L, _, self.H = k_cache.shape
        self.C = K.kv_channels(k_cache, v_cache)   # 1 for a latent (MLA) cache
        self.retention = retention
        self.dev = k_cache.device
        self.on_gpu = self.dev.type == "cuda"
        self.elems = self.C * self.L * page_size * self.H
        self.page_bytes = self.elems * k_cache.element_size()
        self.header = ChunkHeader(chunk_tokens=page_size, block_size=page_size, num_layers=self.L,
                                  hidden_dim=self.H, dtype="bf16", num_kv_channels=self.C)
        dt = k_cache.dtype
        pin = self.on_gpu
        # save ring: slots [head, head + inflight) are in use, released in order;
        # 0 = as many pages as fit in 1 GiB (at least 16)
        n = staging_pages if staging_pages > 0 else max(16, (1 << 30) // self.page_bytes)
        self.n_save = n
        self.save_dev = torch.empty(n, self.elems, dtype=dt, device=self.dev)
        self.save_host = torch.empty(n, self.elems, dtype=dt, pin_memory=pin)
        self.save_host_u8 = self.save_host.view(torch.uint8).numpy()
        self.save_idx_host = torch.zeros(n, dtype=torch.int32, pin_memory=pin)
        self.save_idx_np = self.save_idx_host.numpy()
        self.save_idx_dev = torch.zeros(n, dtype=torch.int32, device=self.dev)
        self.save_head = 0
        self.save_inflight = 0
        self.pending_saves: list[tuple[int, int]] = []
        # promote double buffer
        c = max(1, load_chunk)
        self.load_chunk = c
        self.load_dev = torch.empty(2, c, self.elems, dtype=dt, device=self.dev)
        self.load_host = torch.empty(2, c, self.elems, dtype=dt, pin_memory=pin)
        self.load_host_u8 = self.load_host.view(torch.uint8).numpy()
        self.load_idx_host = torch.zeros(2, c, dtype=torch.int32, pin_memory=pin)
        self.load_idx_np = self.load_idx_host.numpy()
        self.load_idx_dev = torch.zeros(2, c, dtype=torch.int32, device=self.dev)
        self.load_ev = [None, None]
        self.load_buf = 0
        self.async_load = async_load
        self.side = torch.cuda.Stream(self.dev) if self.on_gpu else None
        self.index_sink = None      # fn(kind, Tier, [chained hashes])
        self._lock = threading.Lock()
        self.stats = {"saved": 0, "save_dropped": 0, "save_batches": 0, "promoted": 0, "lookups": 0,
                      "loads": 0, "load_s": 0.0}
        self._save_q: queue.Queue = queue.Queue()
        self.pinned = store if isinstance(store, PinnedPageStore) else None
        if self.pinned is not None:
            self.pinned.bind(self.elems, dt, pin=pin)
        self._writer_t = threading.Thread(target=self._writer, daemon=True, name="kv-tier-writer")
        self._writer_t.start()
        self._load_q: queue.Queue = queue.Queue()
        self._loads_waiting: list = []     # (tag, got, event)
        self._loads_done: queue.Queue = queue.Queue()
        self._new_loads: list = []
        if hasattr(store, "add_listener"):
            store.add_listener(self._on_store_drop)
        # the kvd daemon's shared arena, page-locked: promotes copy pages from
        # it straight into device memory
        self.arena_t = store.register_arena() if self.on_gpu and hasattr(store, "register_arena") else None
        self.stats["direct_pages"] = 0
        self._loader_t = None
        if self.async_load:
            self._loader_t = threading.Thread(target=self._loader, daemon=True, name="kv-tier-loader")
            self._loader_t.start()

    def _key(self, h: int) -> bytes:
        return hash_key(h) + self.key_tag

    def _on_store_drop(self, key: bytes, spilled: bool) -> None:
        """The host store let a block go (to the NVMe tier when spilled)."""
        if self.index_sink is None or len(key) != 8 + len(self.key_tag) or not key.endswith(self.key_tag):
            return
        h = int.from_bytes(key[:8], "little")
        if spilled:     # first: the block keeps a tier, so its index key is kept
            self.index_sink("stored", Tier.DISK, [h])
        self.index_sink("removed", Tier.HOST, [h])

    # ------------------------------------------------------------------ save
    def on_evict(self, page: int, block_hash: int) -> None:
        """The block manager is reusing ``page`` (it held ``block_hash``)."""
        self.pending_saves.append((page, block_hash))

    def flush_saves(self, wait_s: float = 60.0) -> int:
        """Issue the gather + copy-out of every page evicted since the last
        call (call after scheduling, before the forward pass: the pages are
        about to be overwritten). A burst larger than the free staging slots
        goes out in rounds, waiting for the writer to release slots between
        them (backpressure instead of dropping pages); only a writer stuck
        for ``wait_s`` makes the rest count as dropped. Returns the number of
        pages queued."""
        items, self.pending_saves = self.pending_saves, []
        queued = 0
        t0 = time.time()
        while items:
            with self._lock:
                free = self.n_save - self.save_inflight
            if free <= 0:
                if time.time() - t0 > wait_s:
                    break
                time.sleep(0.0005)
                continue
            take, items = items[:free], items[free:]
            self._issue_saves(take)
            queued += len(take)
        self.stats["save_dropped"] += len(items)
        return queued

    def _issue_saves(self, take: list[tuple[int, int]]) -> None:
        arena_slots = None
        if self.pinned is not None:
            res = self.pinned.reserve([self._key(h) for _, h in take])
            kept = [(t, a) for t, a in zip(take, res) if a is not None and a >= 0]
            self.stats["save_dropped"] += sum(1 for a in res if a is not None and a < 0)
            if not kept:
                return
            take = [t for t, _ in kept]
            arena_slots = [a for _, a in kept]
        with self._lock:
            start = self.save_head
            self.save_inflight += len(take)
            self.save_head = (start + len(take)) % self.n_save
        m = len(take)
        slots = [(start + i) % self.n_save for i in range(m)]
        self.save_idx_np[slots] = [p for p, _ in take]
        segs = [(start, min(m, self.n_save - start))]
        if start + m > self.n_save:
            segs.append((0, start + m - self.n_save))
        ev = None
        if self.on_gpu:
            for s0, cnt in segs:
                self.save_idx_dev[s0:s0 + cnt].copy_(self.save_idx_host[s0:s0 + cnt], non_blocking=True)
                K.kv_page_copy(self.k, self.v, self.save_dev[s0:s0 + cnt], self.save_idx_dev[s0:s0 + cnt], self.ps,
                               gather=True, page_major=True)
            gathered = torch.cuda.Event()
            gathered.record()
            with torch.cuda.stream(self.side):
                self.side.wait_event(gathered)
                if arena_slots is None:
                    for s0, cnt in segs:
                        self.save_host[s0:s0 + cnt].copy_(self.save_dev[s0:s0 + cnt], non_blocking=True)
                else:   # straight into the arena slots reserved for the blocks
                    arena = self.pinned.arena
                    for ring, a in zip(slots, arena_slots):
                        arena[a].copy_(self.save_dev[ring], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.side)
        else:
            for s0, cnt in segs:
                K.kv_page_copy(self.k, self.v, self.save_host[s0:s0 + cnt], self.save_idx_host[s0:s0 + cnt],
                               self.ps, gather=True, page_major=True)
            if arena_slots is not None:
                for ring, a in zip(slots, arena_slots):
                    self.pinned.arena[a].copy_(self.save_host[ring])
        self.stats["save_batches"] += 1
        self._save_q.put((slots, [h for _, h in take], ev, arena_slots is not None))

    def _writer(self) -> None:
        while True:
            job = self._save_q.get()
            if job is None:
                return
            slots, hashes, ev, in_arena = job
            if ev is not None:
                ev.synchronize()
            stored = []
            if in_arena:        # the pages already sit in their arena slots
                done = set(self.pinned.commit([self._key(h) for h in hashes]))
                stored = [h for h in hashes if self._key(h) in done]
                self.stats["saved"] += len(stored)
                hashes = []
            for slot, h in zip(slots, hashes):
                try:
                    blob = pack_chunk(self.header, memoryview(self.save_host_u8[slot]))
                    if self.store.set(self._key(h), blob, self.retention):
                        stored.append(h)
                        self.stats["saved"] += 1
                    else:
                        self.stats["save_dropped"] += 1
                except Exception:
                    self.stats["save_dropped"] += 1
            with self._lock:
                self.save_inflight -= len(slots)
            if stored and self.index_sink is not None:
                self.index_sink("stored", Tier.HOST, stored)

    def flush(self, timeout: float = 30.0) -> None:
        """Wait until every queued save has reached the store."""
        self.flush_saves()
        t0 = time.time()
        while True:
            with self._lock:
                busy = self.save_inflight > 0
            if not busy or time.time() - t0 > timeout:
                return
            time.sleep(0.002)

    # ------------------------------------------------------------------ promote
    def match(self, hashes: list[int]) -> int:
        """How many of ``hashes`` (consecutive from the first) a tier holds:
        the external hit count the scheduler accounts for at admission."""
        n = 0
        many = getattr(self.store, "exists_many", None)
        step = 64
        for i in range(0, len(hashes), step):
            part = hashes[i:i + step]
            self.stats["lookups"] += len(part)
            if many is not None:
                hits = many([self._key(h) for h in part])
            else:
                hits = []
                for h in part:
                    ok = self.store.exists(self._key(h))
                    hits.append(ok)
                    if not ok:
                        break
            for ok in hits:
                if not ok:
                    return n
                n += 1
        return n

    def _fill(self, buf: int, pages: list[int], hashes: list[int]) -> int:
        """Read blobs into pinned buffer ``buf``; returns how many consecutive
        pages were filled (a blob that vanished or fails to parse ends it)."""
        m = 0
        read = getattr(self.store, "read", self.store.get)
        for i, (page, h) in enumerate(zip(pages, hashes)):
            blob = read(self._key(h))
            if blob is None:
                break
            try:
                hdr, payload = unpack_chunk(blob)
            except PackedFormatError:
                break
            if (hdr.num_layers != self.L or hdr.hidden_dim != self.H or hdr.chunk_tokens != self.ps
                    or hdr.num_kv_channels != self.C):
                break
            self.load_host_u8[buf, i, :] = np.frombuffer(payload, dtype=np.uint8)
            self.load_idx_np[buf, i] = page
            m += 1
        return m

    def _fill_direct(self, buf: int, pages: list[int], hashes: list[int], stream) -> tuple[int, list]:
        """Arena-resident blobs: one DMA per page from the registered arena
        into the device staging slot. Returns (pages issued, [(arena, blob
        offset, version)]) for the version check after the copies land."""
        from infera_b200.engine.packed_format import unpack_header

        m, checks = 0, []
        for i, (page, h) in enumerate(zip(pages, hashes)):
            r = self.store.read_shared(self._key(h))
            if r is None:
                break
            arena, off, size, ver = r
            try:
                hdr = unpack_header(memoryview(arena.mm)[off:off + min(size, 1 << 16)])
            except PackedFormatError:
                break
            if (hdr.num_layers != self.L or hdr.hidden_dim != self.H or hdr.chunk_tokens != self.ps
                    or hdr.num_kv_channels != self.C or hdr.payload_byte_offset + self.page_bytes > size):
                break
            po = off + hdr.payload_byte_offset
            with torch.cuda.stream(stream):
                self.load_dev[buf, i].view(torch.uint8).copy_(self.arena_t[po:po + self.page_bytes],
                                                             non_blocking=True)
            self.load_idx_np[buf, i] = page
            checks.append((arena, off, ver))
            m += 1
        return m, checks

    def _fill_pinned(self, buf: int, pages: list[int], hashes: list[int], stream) -> int:
        """Arena slots of the leading run of held blocks, copied straight to
        the device staging buffer (one DMA per page) and scattered into the
        pages; the slots stay pinned until the copies have landed."""
        slots = self.pinned.acquire([self._key(h) for h in hashes])
        m = len(slots)
        if not m:
            return 0
        arena = self.pinned.arena
        try:
            if self.on_gpu:
                with torch.cuda.stream(stream):
                    for i, a in enumerate(slots):
                        self.load_dev[buf, i].copy_(arena[a], non_blocking=True)
            else:
                for i, a in enumerate(slots):
                    self.load_host[buf, i].copy_(arena[a])
            self.load_idx_np[buf, :m] = pages[:m]
            self._scatter(buf, m, stream, staged=False)
            self.load_buf ^= 1
            if self.on_gpu:
                self.load_ev[buf].synchronize()
        finally:
            self.pinned.release(slots)
        return m

    def _scatter(self, buf: int, m: int, stream, staged: bool = True) -> None:
        if self.on_gpu:
            with torch.cuda.stream(stream):
                self.load_idx_dev[buf, :m].copy_(self.load_idx_host[buf, :m], non_blocking=True)
                if staged:
                    self.load_dev[buf, :m].copy_(self.load_host[buf, :m], non_blocking=True)
                K.kv_page_copy(self.k, self.v, self.load_dev[buf, :m], self.load_idx_dev[buf, :m], self.ps,
                               gather=False, page_major=True)
                e = torch.cuda.Event()
                e.record(stream)
                self.load_ev[buf] = e
        else:
            K.kv_page_copy(self.k, self.v, self.load_host[buf, :m], self.load_idx_host[buf, :m], self.ps,
                           gather=False, page_major=True)

    def _run_load(self, pages: list[int], hashes: list[int], stream) -> int:
        got = 0
        t0 = time.monotonic()
        for c0 in range(0, len(pages), self.load_chunk):
            buf = self.load_buf
            if self.load_ev[buf] is not None:
                self.load_ev[buf].synchronize()      # that buffer's previous copies have landed
                self.load_ev[buf] = None
            want = pages[c0:c0 + self.load_chunk]
            if self.pinned is not None:
                m = self._fill_pinned(buf, want, hashes[c0:c0 + self.load_chunk], stream)
            elif self.arena_t is not None and hasattr(self.store, "read_shared"):
                m, checks = self._fill_direct(buf, want, hashes[c0:c0 + self.load_chunk], stream)
                if m:
                    self._scatter(buf, m, stream, staged=False)
                    self.load_buf ^= 1
                    # a slot rewritten while it was being copied is not used
                    self.load_ev[buf].synchronize()
                    ok = 0
                    for arena, off, ver in checks:
                        if arena.version_at(off) != ver:
                            break
                        ok += 1
                    self.stats["direct_pages"] += ok
                    m = ok
            else:
                m = self._fill(buf, want, hashes[c0:c0 + self.load_chunk])
                if m:
                    self._scatter(buf, m, stream)
                    self.load_buf ^= 1
            got += m
            if m < len(want):
                break
        self.stats["promoted"] += got
        self.stats["loads"] += 1
        self.stats["load_s"] += time.monotonic() - t0
        return got

    def load(self, pages: list[int], hashes: list[int]) -> int:
        """Synchronous-on-the-host promote (the pages are ready for every
        later kernel of the compute stream when this returns)."""
        stream = torch.cuda.current_stream() if self.on_gpu else None
        return self._run_load(pages, hashes, stream)

    def begin_load(self, tag, pages: list[int], hashes: list[int]) -> None:
        """Queue an asynchronous promote; :meth:`submit_loads` hands it to
        the loader and :meth:`poll_loads` reports it once done."""
        self._new_loads.append((tag, list(pages), list(hashes)))

    def submit_loads(self) -> None:
        """Hand the loads queued by this step to the loader, ordered after
        everything the compute stream has been given so far (the gathers
        that saved these pages' previous content included)."""
        if not self._new_loads:
            return
        jobs, self._new_loads = self._new_loads, []
        after = None
        if self.on_gpu:
            after = torch.cuda.Event()
            after.record()
        if not self.async_load:
            for tag, pages, hashes in jobs:
                self._loads_done.put((tag, self._run_load(pages, hashes, torch.cuda.current_stream()
                                                          if self.on_gpu else None), None))
            return
        for tag, pages, hashes in jobs:
            self._load_q.put((tag, pages, hashes, after))

    def _loader(self) -> None:
        if self.on_gpu:
            torch.cuda.set_device(self.dev)
        while True:
            job = self._load_q.get()
            if job is None:
                return
            tag, pages, hashes, after = job
            try:
                if after is not None:
                    self.side.wait_event(after)
                got = self._run_load(pages, hashes, self.side)
            except Exception:
                got = 0
            done = None
            if self.on_gpu:
                done = torch.cuda.Event()
                done.record(self.side)
            self._loads_done.put((tag, got, done))

    def poll_loads(self) -> list[tuple[object, int]]:
        """Promotes whose copies have completed: [(tag, pages loaded)]."""
        while True:
            try:
                self._loads_waiting.append(self._loads_done.get_nowait())
            except queue.Empty:
                break
        out, keep = [], []
        for tag, got, ev in self._loads_waiting:
            if ev is None or ev.query():
                out.append((tag, got))
            else:
                keep.append((tag, got, ev))
        self._loads_waiting = keep
        return out

    def pending_loads(self) -> int:
        return len(self._new_loads) + self._load_q.qsize() + self._loads_done.qsize() + len(self._loads_waiting)

    def close(self) -> None:
        self._save_q.put(None)
        self._writer_t.join(timeout=10)
        if self._loader_t is not None:
            self._load_q.put(None)
            self._loader_t.join(timeout=10)

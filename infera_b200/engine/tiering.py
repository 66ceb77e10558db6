"""KV-cache tiering for the engine: HBM pages <-> host DRAM <-> NVMe.

* Save on eviction: when the block manager is about to reuse a cached page
  (it held a full, hashed prefix block), the page's K/V (or, for a latent
  MLA cache, its one latent row per token) for every layer is
  gathered on the compute stream into a device staging slot (so the page can
  be overwritten right after), copied to pinned host memory on a side
  stream, and handed to a writer thread that packs it as a v2 KV chunk and
  stores it under the block's chained hash. The host store (the kvd
  ``HostStore``) spills its own evictions to the NVMe tablespace.
* Promote on a prefix hit: after the HBM prefix match, the next consecutive
  block hashes are looked up in the tiers; hits are copied host -> device
  and scattered into freshly allocated pages before the forward pass that
  reads them, and registered in the prefix cache like computed pages. A
  prefix computed on another instance is reusable once it reached a shared
  tier (the daemon's arena / tablespace).

Keys are the 8-byte little-endian chained block hash, so any instance that
computed the same prefix produces the same keys.
"""

from __future__ import annotations

import queue
import threading

import torch

from infera_b200.engine.packed_format import ChunkHeader, PackedFormatError, pack_chunk, unpack_chunk
from infera_b200.ops import kernels as K


def hash_key(h: int) -> bytes:
    return int(h).to_bytes(8, "little", signed=False)


class TierManager:
    def __init__(self, k_cache: torch.Tensor, v_cache: torch.Tensor, store, page_size: int = 16,
                 retention: str = "long", staging_pages: int = 64):
        self.k = k_cache
        self.v = v_cache
        self.store = store
        self.ps = page_size
        self.L, _, self.H = k_cache.shape
        self.C = K.kv_channels(k_cache, v_cache)   # 1 for a latent (MLA) cache
        self.retention = retention
        self.dev = k_cache.device
        self.on_gpu = self.dev.type == "cuda"
        self.page_bytes = self.C * self.L * page_size * self.H * k_cache.element_size()
        self.header = ChunkHeader(chunk_tokens=page_size, block_size=page_size, num_layers=self.L,
                                  hidden_dim=self.H, dtype="bf16", num_kv_channels=self.C)
        n = staging_pages
        self.dev_stage = torch.empty(n, self.C * self.L * page_size * self.H, dtype=k_cache.dtype, device=self.dev)
        self.host_stage = torch.empty(n, self.C * self.L * page_size * self.H, dtype=k_cache.dtype,
                                      pin_memory=self.on_gpu)
        self.free_slots = queue.Queue()
        for i in range(n):
            self.free_slots.put(i)
        self.side = torch.cuda.Stream(self.dev) if self.on_gpu else None
        self.work: queue.Queue = queue.Queue()
        self.stats = {"saved": 0, "save_dropped": 0, "promoted": 0, "lookups": 0}
        self._thread = threading.Thread(target=self._writer, daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------ save
    def on_evict(self, page: int, block_hash: int) -> None:
        try:
            slot = self.free_slots.get_nowait()
        except queue.Empty:
            self.stats["save_dropped"] += 1   # writer is behind: drop, never stall the step
            return
        pages = torch.tensor([page], dtype=torch.int32, device=self.dev)
        K.kv_page_copy(self.k, self.v, self.dev_stage[slot], pages, self.ps, gather=True)
        ev = None
        if self.on_gpu:
            done_gather = torch.cuda.Event()
            done_gather.record()
            with torch.cuda.stream(self.side):
                self.side.wait_event(done_gather)
                self.host_stage[slot].copy_(self.dev_stage[slot], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.side)
        else:
            self.host_stage[slot].copy_(self.dev_stage[slot])
        self.work.put((slot, block_hash, ev))

    def _writer(self) -> None:
        while True:
            slot, h, ev = self.work.get()
            if slot is None:
                return
            if ev is not None:
                ev.synchronize()
            payload = self.host_stage[slot].view(torch.uint8).numpy().tobytes()
            self.free_slots.put(slot)
            try:
                self.store.set(hash_key(h), pack_chunk(self.header, payload), self.retention)
                self.stats["saved"] += 1
            except Exception:
                self.stats["save_dropped"] += 1

    def flush(self, timeout: float = 30.0) -> None:
        """Wait until every queued save has reached the store."""
        import time

        t0 = time.time()
        while not self.work.empty() or self.free_slots.qsize() < self.dev_stage.shape[0]:
            if time.time() - t0 > timeout:
                break
            time.sleep(0.005)

    # ------------------------------------------------------------------ promote
    def match(self, hashes: list[int]) -> int:
        """How many of ``hashes`` (consecutive from the first) a tier holds."""
        n = 0
        for h in hashes:
            self.stats["lookups"] += 1
            if not self.store.exists(hash_key(h)):
                break
            n += 1
        return n

    def load(self, pages: list[int], hashes: list[int]) -> int:
        """Copy the tier copies of ``hashes`` into ``pages``; returns how many
        consecutive pages were filled (a blob that vanished or fails to parse
        ends the run)."""
        done = 0
        for page, h in zip(pages, hashes):
            blob = self.store.get(hash_key(h))
            if blob is None:
                break
            try:
                hdr, payload = unpack_chunk(blob)
            except PackedFormatError:
                break
            if (hdr.num_layers != self.L or hdr.hidden_dim != self.H or hdr.chunk_tokens != self.ps
                    or hdr.num_kv_channels != self.C):
                break
            slot = self.free_slots.get()
            self.host_stage[slot].view(torch.uint8).copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
            self.dev_stage[slot].copy_(self.host_stage[slot], non_blocking=self.on_gpu)
            K.kv_page_copy(self.k, self.v, self.dev_stage[slot], torch.tensor([page], dtype=torch.int32,
                                                                              device=self.dev), self.ps, gather=False)
            if self.on_gpu:
                torch.cuda.current_stream().synchronize()
            self.free_slots.put(slot)
            done += 1
        self.stats["promoted"] += done
        return done

    def close(self) -> None:
        self.work.put((None, None, None))
        self._thread.join(timeout=10)

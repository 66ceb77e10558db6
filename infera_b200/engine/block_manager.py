"""Paged KV-cache block manager with a content-addressed prefix cache.

* A page holds ``page_size`` (16) tokens of K and V for every layer.
* Full pages are content-addressed by the chained block hash
  ``h_i = XXH3_64(h_{i-1} as u64 LE || tokens as u32 LE)`` with
  ``h_{-1} = 0`` - the same chain the router computes from token ids, so an
  engine hash equals the router's hash for the same prefix.
* Pages whose refcount drops to zero keep their hash and sit in an LRU of
  evictable pages; a later request with the same prefix re-references them
  (prefix hit). Allocation takes never-hashed free pages first, then evicts
  the least recently used cached page.
* Every page that becomes cached is reported as ``BlockStored`` and every
  eviction as ``BlockRemoved`` through the ``event_sink`` callback, in the
  vLLM KV-event vocabulary the router consumes.

Reference parity: the reference leaves paging to its engines (vLLM's
KVCacheManager / SGLang's RadixCache); its router-side mirror of this cache
is ``infera/router/kv_event/client.py`` and the hash chain
``infera/router/kv_event/hasher.py:20-42``.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Callable

from infera_b200.utils.hashing import chain_hashes


@dataclass
class SeqBlocks:
    """Per-sequence page list and how many of its tokens are in the cache."""

    pages: list[int] = field(default_factory=list)
    hashes: list[int] = field(default_factory=list)   # hashes of the full pages registered so far
    num_cached_tokens: int = 0                          # tokens with K/V present (computed or hit)
    # (first page, page count) that a KV tier holds and an asynchronous
    # promote will fill; the scheduler parks the sequence until it lands
    tier_load: tuple[int, int] | None = None
    # free pages set aside for this sequence's next pages: the rest of the
    # 8-page tile its last page started, so the tile is one consecutive run
    run_ahead: list[int] = field(default_factory=list)


class BlockManager:
    def __init__(self, num_pages: int, page_size: int = 16, enable_prefix_cache: bool = True,
                 event_sink: Callable[[str, dict], None] | None = None, reserved_pages: int = 1):
        self.num_pages = num_pages
        self.page_size = page_size
        self.enable_prefix_cache = enable_prefix_cache
        self.event_sink = event_sink
        # page 0.. reserved_pages-1 are never handed out (padding target for graphs)
        self.reserved = reserved_pages
        self.refcount = [0] * num_pages
        self.page_hash: list[int | None] = [None] * num_pages
        # free never-hashed pages: a stack (lazily cleaned) plus the set that
        # says which entries are still free; a sequence's next page is its
        # last page + 1 when that one is free, so sequences hold runs of
        # consecutive pages (the decode attention loads an 8-page run as one
        # TMA box per half)
        self.free_plain: list[int] = list(range(num_pages - 1, reserved_pages - 1, -1))
        self.free_set: set[int] = set(self.free_plain)
        self.evictable: OrderedDict[int, None] = OrderedDict()   # cached pages with refcount 0 (LRU order)
        self.hash_to_page: dict[int, int] = {}
        self.stats = {"hit_tokens": 0, "query_tokens": 0, "evictions": 0, "tier_hit_tokens": 0}
        self.tier = None   # optional TierManager: saves evicted prefix pages, promotes them back

    # ------------------------------------------------------------------ capacity
    def num_free(self) -> int:
        return len(self.free_set) + len(self.evictable)

    def usage(self) -> float:
        usable = self.num_pages - self.reserved
        return 1.0 - self.num_free() / max(1, usable)

    def can_allocate(self, n: int, watermark: int = 0) -> bool:
        return self.num_free() - watermark >= n

    # ------------------------------------------------------------------ allocation
    def _push_free(self, page: int) -> None:
        if page not in self.free_set:
            self.free_set.add(page)
            self.free_plain.append(page)
            if len(self.free_plain) > 2 * len(self.free_set) + 1024:
                # drop stale entries (pages taken as a run's next page),
                # keeping each free page's latest position in the stack
                seen: set[int] = set()
                keep = []
                for q in reversed(self.free_plain):
                    if q in self.free_set and q not in seen:
                        seen.add(q)
                        keep.append(q)
                self.free_plain = keep[::-1]

    # pages per attention key tile: a tile of consecutive pages loads as one
    # TMA box per 64-dim half
    RUN = 8

    def _take_run_page(self, sb: SeqBlocks) -> int:
        """The sequence's next page. At the start of an 8-page key tile the
        seven pages after the one taken are set aside for the same sequence
        when they are free, so sequences that grow side by side (decode
        steps) still fill each tile with one run of consecutive pages."""
        if sb.run_ahead:
            return sb.run_ahead.pop(0)
        p = self._take_page(sb.pages[-1] if sb.pages else None)
        if len(sb.pages) % self.RUN == 0 and len(self.free_set) > 64 * self.RUN:
            run = [p + i for i in range(1, self.RUN)]
            if all(q in self.free_set for q in run):
                for q in run:
                    self.free_set.discard(q)      # their stack entries are skipped when reached
                sb.run_ahead = run
        return p

    def _drop_run_ahead(self, sb: SeqBlocks) -> None:
        for q in sb.run_ahead:
            self._push_free(q)
        sb.run_ahead = []

    def _take_page(self, prev: int | None = None) -> int:
        if prev is not None and prev + 1 in self.free_set:
            self.free_set.discard(prev + 1)      # its stack entry is skipped when reached
            return prev + 1
        while self.free_plain:
            page = self.free_plain.pop()
            if page in self.free_set:
                self.free_set.discard(page)
                return page
        if not self.evictable:
            raise MemoryError("KV cache exhausted")
        page, _ = self.evictable.popitem(last=False)
        h = self.page_hash[page]
        if h is not None:
            if self.tier is not None:
                self.tier.on_evict(page, h)   # copy out before the page is reused
            if self.hash_to_page.get(h) == page:
                del self.hash_to_page[h]
            self.page_hash[page] = None
            self.stats["evictions"] += 1
            self._emit("BlockRemoved", {"block_hashes": [h], "medium": "GPU"})
        return page

    def _release(self, page: int) -> None:
        self.refcount[page] -= 1
        if self.refcount[page] == 0:
            if self.page_hash[page] is not None and self.enable_prefix_cache:
                self.evictable[page] = None
            else:
                self.page_hash[page] = None
                self._push_free(page)

    def _emit(self, kind: str, payload: dict) -> None:
        if self.event_sink is not None:
            self.event_sink(kind, payload)

    # ------------------------------------------------------------------ prefix lookup
    def match_prefix(self, token_ids: list[int], hashes: list[int] | None = None) -> tuple[list[int], list[int]]:
        """Longest run of cached full pages at the start of ``token_ids``.

        Returns (pages, hashes) of the hit; at least one token is always left
        to compute, so a fully cached prompt gives back its last page.
        """
        if not self.enable_prefix_cache:
            return [], []
        if hashes is None:
            hashes = chain_hashes(token_ids, self.page_size)
        pages: list[int] = []
        for h in hashes:
            p = self.hash_to_page.get(h)
            if p is None:
                break
            pages.append(p)
        n = len(pages)
        if n > 0 and n * self.page_size >= len(token_ids):
            n -= 1
        return pages[:n], hashes[:n]

    def allocate_prompt(self, token_ids: list[int], num_tokens: int,
                        hashes: list[int] | None = None) -> SeqBlocks | None:
        """Reference the prefix hit and allocate pages for ``num_tokens``
        tokens in total. Returns None (and changes nothing) if memory is
        short."""
        if hashes is None:
            hashes = chain_hashes(token_ids, self.page_size)
        hit_pages, hit_hashes = self.match_prefix(token_ids, hashes)
        n_tier = 0
        if self.tier is not None and self.enable_prefix_cache:
            n_tier = self.tier.match(hashes[len(hit_pages):])
            if (len(hit_pages) + n_tier) * self.page_size >= len(token_ids):
                n_tier = max(0, (len(token_ids) - 1) // self.page_size - len(hit_pages))
        need = (num_tokens + self.page_size - 1) // self.page_size - len(hit_pages)
        # hit pages that are currently evictable do not count as free for us
        hit_evictable = sum(1 for p in hit_pages if self.refcount[p] == 0)
        if self.num_free() - hit_evictable < need:
            return None
        for p in hit_pages:
            if self.refcount[p] == 0:
                self.evictable.pop(p, None)
            self.refcount[p] += 1
        sb = SeqBlocks(pages=list(hit_pages), hashes=list(hit_hashes),
                       num_cached_tokens=len(hit_pages) * self.page_size)
        for _ in range(max(0, need)):
            p = self._take_run_page(sb)
            self.refcount[p] = 1
            sb.pages.append(p)
        if n_tier > 0:
            start = len(hit_pages)
            if getattr(self.tier, "async_load", False):
                sb.tier_load = (start, n_tier)
            else:
                got = self.tier.load(sb.pages[start:start + n_tier], hashes[start:start + n_tier])
                if got > 0:
                    self.commit_full_pages(sb, token_ids, (start + got) * self.page_size)
                    sb.num_cached_tokens = (start + got) * self.page_size
                    self.stats["tier_hit_tokens"] += got * self.page_size
        self.stats["hit_tokens"] += sb.num_cached_tokens
        self.stats["query_tokens"] += len(token_ids)
        return sb

    def ensure_capacity(self, sb: SeqBlocks, num_tokens: int) -> bool:
        """Grow ``sb`` to hold ``num_tokens`` tokens; False if memory is short."""
        need = (num_tokens + self.page_size - 1) // self.page_size - len(sb.pages)
        if need <= 0:
            return True
        if self.num_free() + len(sb.run_ahead) < need:
            return False
        for _ in range(need):
            p = self._take_run_page(sb)
            self.refcount[p] = 1
            sb.pages.append(p)
        return True

    def commit_full_pages(self, sb: SeqBlocks, token_ids: list[int], num_computed: int) -> None:
        """Register every page that is now completely computed in the prefix
        cache (and announce it)."""
        sb.num_cached_tokens = max(sb.num_cached_tokens, num_computed)
        if not self.enable_prefix_cache:
            return
        n_full = num_computed // self.page_size
        start = len(sb.hashes)
        if n_full <= start:
            return
        parent = sb.hashes[-1] if sb.hashes else 0
        new_hashes = chain_hashes(token_ids[start * self.page_size: n_full * self.page_size], self.page_size,
                                  parent=parent)
        stored_h: list[int] = []
        stored_tokens: list[int] = []
        first_parent = parent
        for i, h in enumerate(new_hashes):
            idx = start + i
            page = sb.pages[idx]
            sb.hashes.append(h)
            existing = self.hash_to_page.get(h)
            if existing is None:
                self.hash_to_page[h] = page
                self.page_hash[page] = h
                stored_h.append(h)
                stored_tokens.extend(token_ids[idx * self.page_size:(idx + 1) * self.page_size])
            elif existing != page:
                # identical content computed twice (two requests raced on the
                # same prefix); keep the first copy, this page stays private
                pass
        if stored_h:
            self._emit("BlockStored", {
                "block_hashes": stored_h,
                "parent_block_hash": first_parent if start > 0 else None,
                "token_ids": stored_tokens,
                "block_size": self.page_size,
                "lora_id": None,
                "medium": "GPU",
            })

    def free(self, sb: SeqBlocks) -> None:
        self._drop_run_ahead(sb)
        # release in reverse so the tail of a prefix is evicted before its head
        for p in reversed(sb.pages):
            self._release(p)
        sb.pages = []
        sb.hashes = []

    def clear_cache(self) -> None:
        """Drop every evictable cached page (AllBlocksCleared)."""
        for page in list(self.evictable.keys()):
            h = self.page_hash[page]
            if h is not None and self.hash_to_page.get(h) == page:
                del self.hash_to_page[h]
            self.page_hash[page] = None
            self._push_free(page)
        self.evictable.clear()
        self._emit("AllBlocksCleared", {})

    def cached_hashes(self) -> list[int]:
        return list(self.hash_to_page.keys())

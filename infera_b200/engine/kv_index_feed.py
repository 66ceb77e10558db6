"""Engine-side publisher of the tier-aware KV index (the router's Phase-1
index: which prefixes an instance holds in GPU memory, pinned host memory
or on disk).

The engine's block manager announces device blocks as vLLM-style
``BlockStored`` / ``BlockRemoved`` / ``AllBlocksCleared`` events keyed by
the router's seed-0 chain hash; the tier manager announces the same blocks
entering or leaving the host and disk tiers. This feed translates both into
the index's own keys (``infera_b200.kv.hashing``: seed-1337 content hash +
sequence chain) and batches them as ``EventBatch`` es for a
:class:`~infera_b200.kv.publisher.KvIndexPublisher` (ZMQ PUB, topic
``kv-index``). It keeps what it announced in a local index, from which
:meth:`snapshot` answers the router's reconciler.

A block's index key is derived once, when the device stores it (its
tokens and its parent are known then), and kept while any tier holds the
block. Role of the reference's engine-side probe + publisher
(``infera/kv/probe.py:43-244``, ``infera/kv/publisher.py:46``).
"""

from __future__ import annotations

import threading

from infera_b200.kv.hashing import hash_token_blocks
from infera_b200.kv.index import KVIndex
from infera_b200.kv.types import BlockKey, Tier
from infera_b200.kv.wire import EventBatch, NormalizedEvent, snapshot_json


class KvIndexFeed:
    def __init__(self, publisher: str, model: str, compat: str, page_size: int, sink=None):
        self.publisher, self.model, self.compat = publisher, model, compat
        self.ps = page_size
        self.sink = sink                       # fn(EventBatch)
        self._key = (model, compat, publisher)
        self._local = KVIndex()
        # router chain hash -> [index key, index parent sequence hash, tiers]
        self._blocks: dict[int, list] = {}
        self._pending: list[NormalizedEvent] = []
        self._lock = threading.Lock()
        self.published_batches = 0

    # ------------------------------------------------------------------ inputs
    def on_engine_event(self, kind: str, payload: dict) -> None:
        """The block manager's event (device tier)."""
        with self._lock:
            if kind == "BlockStored":
                self._stored_device(payload)
            elif kind == "BlockRemoved":
                self._removed([int(h) for h in payload.get("block_hashes", [])], Tier.DEVICE)
            elif kind == "AllBlocksCleared":
                for h in [h for h, b in self._blocks.items() if Tier.DEVICE in b[2]]:
                    self._drop_tier(h, Tier.DEVICE)
                self._local.clear(self._key, Tier.DEVICE)
                self._pending.append(NormalizedEvent("cleared", Tier.DEVICE))

    def on_tier_event(self, kind: str, tier: Tier, router_hashes: list[int]) -> None:
        """``kind`` "stored" / "removed": the tier manager saved these blocks
        to (or lost them from) ``tier``."""
        with self._lock:
            if kind == "stored":
                for h in router_hashes:
                    b = self._blocks.get(int(h))
                    if b is None:       # never announced on the device (key unknown): skip
                        continue
                    b[2].add(tier)
                    self._local.apply_stored(self._key, [b[0]], b[1], tier)
                    self._pending.append(NormalizedEvent("stored", tier, [b[0]], b[1]))
            elif kind == "removed":
                self._removed([int(h) for h in router_hashes], tier)

    def _stored_device(self, payload: dict) -> None:
        hashes = [int(h) for h in payload.get("block_hashes", [])]
        toks = payload.get("token_ids") or []
        parent = payload.get("parent_block_hash")
        if not hashes or len(toks) < len(hashes) * self.ps:
            return
        pseq = 0
        if parent is not None:
            pb = self._blocks.get(int(parent))
            if pb is None:
                return          # the parent's key is unknown: the reconciler repairs this
            pseq = pb[0].sequence_hash
        keys = hash_token_blocks(toks[: len(hashes) * self.ps], self.ps, parent_sequence_hash=pseq)
        run: list[BlockKey] = []
        par = pseq or None
        for h, k in zip(hashes, keys):
            b = self._blocks.get(h)
            if b is None:
                self._blocks[h] = [k, par, {Tier.DEVICE}]
            else:
                b[2].add(Tier.DEVICE)
            run.append(k)
            par = k.sequence_hash
        self._local.apply_stored(self._key, run, pseq or None, Tier.DEVICE)
        self._pending.append(NormalizedEvent("stored", Tier.DEVICE, run, pseq or None))

    def _drop_tier(self, h: int, tier: Tier) -> BlockKey | None:
        b = self._blocks.get(h)
        if b is None:
            return None
        b[2].discard(tier)
        if not b[2]:
            del self._blocks[h]
        return b[0]

    def _removed(self, hashes: list[int], tier: Tier) -> None:
        gone = []
        for h in hashes:
            k = self._drop_tier(h, tier)
            if k is not None:
                gone.append(k.sequence_hash)
        if gone:
            self._local.apply_removed(self._key, gone, tier)
            self._pending.append(NormalizedEvent("removed", tier, removed=gone))

    # ------------------------------------------------------------------ outputs
    def flush(self) -> EventBatch | None:
        with self._lock:
            if not self._pending:
                return None
            b = EventBatch(self.publisher, self.model, self.compat, self._pending)
            self._pending = []
        if self.sink is not None:
            self.sink(b)
        self.published_batches += 1
        return b

    def snapshot(self) -> dict:
        with self._lock:
            return snapshot_json(self.publisher, self.model, self.compat, self._local.chains(self._key))

    def tiers_of(self, router_hash: int) -> set:
        with self._lock:
            b = self._blocks.get(int(router_hash))
            return set(b[2]) if b is not None else set()

"""Engine-agnostic probe: turns an engine's block callbacks into index
events.

An engine caches blocks of ``engine_block`` tokens; the index hashes blocks
of ``index_block`` tokens (a multiple). The probe is told, per sequence,
which engine blocks became resident (with their tokens) and which were
evicted, and keeps per-sequence state so that:

* index block ``i`` is announced stored once all its engine blocks are
  resident (the run continues from the previous index block's sequence
  hash, so events chain);
* evicting any engine block of an index block announces that index block
  (and, through the tree, everything after it) removed.

It also keeps what it announced, so a snapshot can be produced from it.
Role of ``infera/kv/probe.py:43-244``.
"""

from __future__ import annotations

from infera_b200.kv.hashing import hash_token_blocks
from infera_b200.kv.index import KVIndex
from infera_b200.kv.types import BlockKey, Tier
from infera_b200.kv.wire import EventBatch, NormalizedEvent


class KvEventProbe:
    def __init__(self, publisher: str, model: str, compat: str, engine_block: int, index_block: int,
                 tier: Tier = Tier.DEVICE, sink=None):
        if index_block % engine_block:
            raise ValueError("index block must be a multiple of the engine block")
        self.publisher, self.model, self.compat = publisher, model, compat
        self.eb, self.ib = engine_block, index_block
        self.tier = tier
        self.sink = sink                     # fn(EventBatch)
        self._pending: list[NormalizedEvent] = []
        # announced state: sequence hash -> BlockKey, for snapshots
        self._local = KVIndex()
        self._key = (model, compat, publisher)
        # engine block hash -> (sequence_hash of the index block containing it)
        self._owner: dict[int, int] = {}

    def on_sequence_cached(self, tokens: list[int], engine_block_hashes: list[int]) -> None:
        """``tokens``: the sequence's tokens covering every resident engine
        block (``len(engine_block_hashes) * engine_block``)."""
        n_ib = (len(engine_block_hashes) * self.eb) // self.ib
        keys = hash_token_blocks(tokens[: n_ib * self.ib], self.ib)
        per = self.ib // self.eb
        new_from = None
        for i, k in enumerate(keys):
            for eh in engine_block_hashes[i * per:(i + 1) * per]:
                self._owner[eh] = k.sequence_hash
            if self._local._tree(self._key).by_seq.get(k.sequence_hash) is None and new_from is None:
                new_from = i
        if new_from is None:
            return
        parent = keys[new_from - 1].sequence_hash if new_from > 0 else None
        run = keys[new_from:]
        self._local.apply_stored(self._key, run, parent, self.tier)
        self._pending.append(NormalizedEvent("stored", self.tier, run, parent))

    def on_engine_blocks_evicted(self, engine_block_hashes: list[int]) -> None:
        gone = []
        for eh in engine_block_hashes:
            s = self._owner.pop(eh, None)
            if s is not None and s not in gone:
                gone.append(s)
        if gone:
            self._local.apply_removed(self._key, gone, None)
            self._pending.append(NormalizedEvent("removed", self.tier, removed=gone))

    def on_cleared(self) -> None:
        self._local.clear(self._key)
        self._owner.clear()
        self._pending.append(NormalizedEvent("cleared", self.tier))

    def flush(self) -> EventBatch | None:
        if not self._pending:
            return None
        b = EventBatch(self.publisher, self.model, self.compat, self._pending)
        self._pending = []
        if self.sink is not None:
            self.sink(b)
        return b

    def chains(self) -> list[tuple[list[BlockKey], Tier]]:
        return self._local.chains(self._key)

"""The tier-aware KV index: one radix tree per (model, compat_key, publisher).

A node is one cached block of one publisher, reached from the root by the
blocks before it (children keyed by ``block_hash``; the node also keeps its
``sequence_hash``, so removals by sequence hash find it through a side
map). A node records the tiers the publisher holds it in. ``find_matches``
walks a query's blocks down every publisher's tree and reports, per tier,
the length of the leading run held in that tier or a faster one.

Routing may place *optimistic* nodes (the block will exist on the chosen
publisher once its request runs) with a deadline; a real stored event
confirms them, ``evict_expired`` drops the unconfirmed.

Methods are synchronous; one writer applies events (``KvIndexWriter``) and
readers run on the same event loop. Semantics of ``infera/kv/index.py:73-454``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

from infera_b200.kv.types import BlockKey, OverlapBlocks, Tier

IndexKey = tuple[str, str, str]  # (model, compat_key, publisher)


def now_ms() -> int:
    return int(time.monotonic() * 1000)


@dataclass
class Node:
    block_hash: int
    sequence_hash: int
    parent: "Node | None" = None
    children: dict[int, "Node"] = field(default_factory=dict)
    tiers: set[Tier] = field(default_factory=set)
    inserted_ms: int = 0
    accessed_ms: int = 0
    optimistic_until_ms: int | None = None


@dataclass
class IndexStats:
    trees: int = 0
    nodes: int = 0
    optimistic: int = 0
    stored_events: int = 0
    removed_events: int = 0
    dropped_unknown_parent: int = 0


class _Tree:
    def __init__(self) -> None:
        self.root = Node(0, 0)
        self.by_seq: dict[int, Node] = {}

    def remove_subtree(self, node: Node) -> int:
        n = 0
        stack = [node]
        while stack:
            x = stack.pop()
            stack.extend(x.children.values())
            self.by_seq.pop(x.sequence_hash, None)
            n += 1
        if node.parent is not None:
            node.parent.children.pop(node.block_hash, None)
        return n


class KVIndex:
    def __init__(self) -> None:
        self._trees: dict[IndexKey, _Tree] = {}
        self.stats = IndexStats()

    def _tree(self, key: IndexKey, create: bool = True) -> _Tree | None:
        t = self._trees.get(key)
        if t is None and create:
            t = self._trees[key] = _Tree()
        return t

    def drop_publisher(self, publisher: str) -> int:
        """Forget every tree of ``publisher`` (it left the fleet)."""
        keys = [k for k in self._trees if k[2] == publisher]
        for k in keys:
            del self._trees[k]
        return len(keys)

    def tier_counts(self, publisher: str) -> dict[str, int]:
        """Blocks ``publisher`` holds per tier (over all its trees)."""
        out: dict[str, int] = {}
        for k, t in self._trees.items():
            if k[2] != publisher:
                continue
            for node in t.by_seq.values():
                for tier in node.tiers:
                    out[tier.value] = out.get(tier.value, 0) + 1
        return out

    def publishers(self, model: str, compat: str) -> list[str]:
        return [k[2] for k in self._trees if k[0] == model and k[1] == compat]

    # ------------------------------------------------------------------ writes
    def apply_stored(self, key: IndexKey, blocks: list[BlockKey], parent_sequence_hash: int | None = None,
                     tier: Tier = Tier.DEVICE, ts_ms: int | None = None) -> int:
        """Blocks stored consecutively after ``parent_sequence_hash`` (None:
        from the root). Returns how many nodes were added or updated."""
        t = self._tree(key)
        ts = now_ms() if ts_ms is None else ts_ms
        if parent_sequence_hash in (None, 0):
            cur = t.root
        else:
            cur = t.by_seq.get(parent_sequence_hash)
            if cur is None:
                self.stats.dropped_unknown_parent += 1
                return 0
        n = 0
        for b in blocks:
            nxt = cur.children.get(b.block_hash)
            if nxt is None or nxt.sequence_hash != b.sequence_hash:
                if nxt is not None:
                    t.remove_subtree(nxt)
                nxt = Node(b.block_hash, b.sequence_hash, parent=cur, inserted_ms=ts)
                cur.children[b.block_hash] = nxt
                t.by_seq[b.sequence_hash] = nxt
            nxt.tiers.add(tier)
            nxt.optimistic_until_ms = None
            nxt.accessed_ms = ts
            cur = nxt
            n += 1
        self.stats.stored_events += 1
        return n

    def apply_removed(self, key: IndexKey, sequence_hashes: list[int], tier: Tier | None = None) -> int:
        """Drop the blocks from ``tier`` (all tiers if None). A block left in
        no tier is removed with its subtree (its descendants are unreachable
        as prefixes)."""
        t = self._tree(key, create=False)
        if t is None:
            return 0
        n = 0
        for s in sequence_hashes:
            node = t.by_seq.get(s)
            if node is None:
                continue
            if tier is None:
                node.tiers.clear()
            else:
                node.tiers.discard(tier)
            if not node.tiers:
                n += t.remove_subtree(node)
        self.stats.removed_events += 1
        return n

    def clear(self, key: IndexKey, tier: Tier | None = None) -> None:
        t = self._tree(key, create=False)
        if t is None:
            return
        if tier is None:
            del self._trees[key]
            return
        for node in list(t.by_seq.values()):
            node.tiers.discard(tier)
        for node in list(t.root.children.values()):
            self._prune(t, node)

    def _prune(self, t: _Tree, node: Node) -> None:
        if not node.tiers and node.optimistic_until_ms is None:
            t.remove_subtree(node)
            return
        for c in list(node.children.values()):
            self._prune(t, c)

    def insert_optimistic(self, key: IndexKey, blocks: list[BlockKey], ttl_ms: int = 10_000,
                          tier: Tier = Tier.DEVICE) -> int:
        t = self._tree(key)
        until = now_ms() + ttl_ms
        cur = t.root
        n = 0
        for b in blocks:
            nxt = cur.children.get(b.block_hash)
            if nxt is None:
                nxt = Node(b.block_hash, b.sequence_hash, parent=cur, inserted_ms=now_ms(),
                           optimistic_until_ms=until)
                nxt.tiers.add(tier)
                cur.children[b.block_hash] = nxt
                t.by_seq[b.sequence_hash] = nxt
                n += 1
            cur = nxt
        return n

    def evict_expired(self, now: int | None = None) -> int:
        now = now_ms() if now is None else now
        n = 0
        for t in self._trees.values():
            for node in [x for x in t.by_seq.values() if x.optimistic_until_ms is not None
                         and x.optimistic_until_ms < now]:
                if node.sequence_hash in t.by_seq:
                    n += t.remove_subtree(node)
        return n

    def replace(self, key: IndexKey, chains: list[tuple[list[BlockKey], Tier]]) -> None:
        """Reset one publisher's tree to a snapshot (reconciliation)."""
        self._trees.pop(key, None)
        for blocks, tier in chains:
            self.apply_stored(key, blocks, None, tier)

    # ------------------------------------------------------------------ reads
    def find_matches(self, model: str, compat: str, query: list[BlockKey]) -> dict[str, OverlapBlocks]:
        out: dict[str, OverlapBlocks] = {}
        ts = now_ms()
        for key, t in self._trees.items():
            if key[0] != model or key[1] != compat:
                continue
            ob = OverlapBlocks(key[2])
            best_rank = -1  # slowest tier needed so far along the run
            cur = t.root
            for i, b in enumerate(query):
                nxt = cur.children.get(b.block_hash)
                if nxt is None or nxt.sequence_hash != b.sequence_hash or not nxt.tiers:
                    break
                nxt.accessed_ms = ts
                fastest = min(x.rank for x in nxt.tiers)
                best_rank = max(best_rank, fastest)
                for tier in Tier:
                    if tier.rank >= best_rank:
                        ob.by_tier[tier] = i + 1
                cur = nxt
            if ob.by_tier:
                out[key[2]] = ob
        return out

    def size(self) -> IndexStats:
        s = IndexStats(trees=len(self._trees), stored_events=self.stats.stored_events,
                       removed_events=self.stats.removed_events,
                       dropped_unknown_parent=self.stats.dropped_unknown_parent)
        for t in self._trees.values():
            s.nodes += len(t.by_seq)
            s.optimistic += sum(1 for x in t.by_seq.values() if x.optimistic_until_ms is not None)
        return s

    def chains(self, key: IndexKey) -> list[tuple[list[BlockKey], Tier]]:
        """What a snapshot carries: for every tier, the root-to-leaf chains
        of blocks that all hold that tier (a block in two tiers appears in a
        chain of each; replaying the chains restores every node's tiers)."""
        t = self._trees.get(key)
        if t is None:
            return []
        out = []
        for tier in Tier:
            stack = [(c, [c]) for c in t.root.children.values() if tier in c.tiers]
            while stack:
                node, path = stack.pop()
                kids = [c for c in node.children.values() if tier in c.tiers]
                if not kids:
                    out.append(([BlockKey(x.block_hash, x.sequence_hash) for x in path], tier))
                for c in kids:
                    stack.append((c, path + [c]))
        return out

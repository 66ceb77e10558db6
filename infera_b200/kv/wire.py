"""Wire formats of the tier-aware KV index.

* ``EventBatch`` (msgpack, ZMQ multipart ``[b"kv-index", seq u64 BE,
  batch]``): ``{"v": 1, "publisher", "model", "compat", "ts",
  "events": [NormalizedEvent]}`` with each event
  ``{"k": "stored"|"removed"|"cleared", "tier", "parent", "blocks":
  [[block_hash, sequence_hash], ...]}`` (removed events carry sequence
  hashes in ``blocks``).
* ``Snapshot`` (JSON over HTTP ``GET /v1/kv-index/snapshot``): the
  publisher's chains ``{"publisher", "model", "compat", "ts", "chains":
  [{"tier", "blocks": [[bh, sh], ...]}]}``; hashes are decimal strings in
  JSON (they exceed 2^53).

Role of ``infera/kv/wire.py:27-339`` (this framework's own schema).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import msgpack

from infera_b200.kv.types import BlockKey, Tier

TOPIC = b"kv-index"
VERSION = 1


@dataclass
class NormalizedEvent:
    kind: str                      # stored / removed / cleared
    tier: Tier = Tier.DEVICE
    blocks: list[BlockKey] = field(default_factory=list)
    parent: int | None = None      # sequence hash the stored run continues
    removed: list[int] = field(default_factory=list)


@dataclass
class EventBatch:
    publisher: str
    model: str
    compat: str
    events: list[NormalizedEvent]
    ts: float = field(default_factory=time.time)


def encode_batch(b: EventBatch) -> bytes:
    evs = []
    for e in b.events:
        d = {"k": e.kind, "tier": e.tier.value}
        if e.kind == "stored":
            d["parent"] = e.parent
            d["blocks"] = [[x.block_hash, x.sequence_hash] for x in e.blocks]
        elif e.kind == "removed":
            d["blocks"] = list(e.removed)
        evs.append(d)
    return msgpack.packb({"v": VERSION, "publisher": b.publisher, "model": b.model, "compat": b.compat,
                          "ts": b.ts, "events": evs}, use_bin_type=True)


def decode_batch(raw: bytes) -> EventBatch:
    d = msgpack.unpackb(raw, raw=False)
    if d.get("v") != VERSION:
        raise ValueError(f"unsupported kv-index batch version {d.get('v')!r}")
    evs = []
    for e in d["events"]:
        tier = Tier(e.get("tier", "device"))
        if e["k"] == "stored":
            evs.append(NormalizedEvent("stored", tier, [BlockKey(int(a), int(b)) for a, b in e["blocks"]],
                                       e.get("parent")))
        elif e["k"] == "removed":
            evs.append(NormalizedEvent("removed", tier, removed=[int(x) for x in e["blocks"]]))
        elif e["k"] == "cleared":
            evs.append(NormalizedEvent("cleared", tier))
    return EventBatch(d["publisher"], d["model"], d["compat"], evs, d.get("ts", 0.0))


def snapshot_json(publisher: str, model: str, compat: str, chains: list[tuple[list[BlockKey], Tier]]) -> dict:
    return {"publisher": publisher, "model": model, "compat": compat, "ts": time.time(),
            "chains": [{"tier": t.value, "blocks": [[str(b.block_hash), str(b.sequence_hash)] for b in bl]}
                       for bl, t in chains]}


def snapshot_chains(d: dict) -> list[tuple[list[BlockKey], Tier]]:
    return [([BlockKey(int(a), int(b)) for a, b in c["blocks"]], Tier(c.get("tier", "device")))
            for c in d.get("chains", [])]

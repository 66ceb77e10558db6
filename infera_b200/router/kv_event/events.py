"""KV-event wire schemas.

Two encodings exist in the fleet and both are decoded:

* vLLM: a batch ``[ts, [event, ...], attn_dp_rank]`` whose events are tagged
  MAPS (``{"type": "BlockStored", ...}``); hashes are int or bytes.
* SGLang: the same batch shape with tagged ARRAY events.

This framework's engine publishes the vLLM map encoding. The field names and
tags are a wire contract with the engines (``infera/router/kv_event/events.py:34-142``).
"""

from __future__ import annotations

import msgspec


class _MapEvent(msgspec.Struct, omit_defaults=True, gc=False, tag=True):
    pass


class BlockStored(_MapEvent):
    block_hashes: list[int | bytes]
    parent_block_hash: int | bytes | None
    token_ids: list[int]
    block_size: int
    lora_id: int | None
    medium: str | None = None
    group_idx: int | None = None
    kv_cache_spec_kind: str | None = None


class BlockRemoved(_MapEvent):
    block_hashes: list[int | bytes]
    medium: str | None = None


class AllBlocksCleared(_MapEvent):
    pass


class KVEventBatch(msgspec.Struct, array_like=True, omit_defaults=True, gc=False):
    ts: float
    events: list[BlockStored | BlockRemoved | AllBlocksCleared]
    attn_dp_rank: int | None = None


class _ArrEvent(msgspec.Struct, array_like=True, omit_defaults=True, gc=False, tag=True):
    pass


class SgBlockStored(_ArrEvent, tag="BlockStored"):
    block_hashes: list[int]
    parent_block_hash: int | None
    token_ids: list[int]
    block_size: int
    lora_id: int | None = None


class SgBlockRemoved(_ArrEvent, tag="BlockRemoved"):
    block_hashes: list[int]


class SgAllBlocksCleared(_ArrEvent, tag="AllBlocksCleared"):
    pass


class SgKVEventBatch(msgspec.Struct, array_like=True, omit_defaults=True, gc=False):
    ts: float
    events: list[SgBlockStored | SgBlockRemoved | SgAllBlocksCleared]
    attn_dp_rank: int | None = None


STORED = (BlockStored, SgBlockStored)
REMOVED = (BlockRemoved, SgBlockRemoved)
CLEARED = (AllBlocksCleared, SgAllBlocksCleared)

_ENCODER = msgspec.msgpack.Encoder()


def batch_type_for_engine(engine: str):
    return SgKVEventBatch if engine == "sglang" else KVEventBatch


def decoder_for_engine(engine: str) -> msgspec.msgpack.Decoder:
    return msgspec.msgpack.Decoder(type=batch_type_for_engine(engine))


def encode_batch(batch: KVEventBatch) -> bytes:
    return _ENCODER.encode(batch)


def event_from_dict(kind: str, payload: dict):
    """Build a vLLM-encoding event from the engine's (kind, payload) callback."""
    if kind == "BlockStored":
        return BlockStored(block_hashes=list(payload["block_hashes"]),
                           parent_block_hash=payload.get("parent_block_hash"),
                           token_ids=list(payload["token_ids"]), block_size=int(payload["block_size"]),
                           lora_id=payload.get("lora_id"), medium=payload.get("medium"),
                           kv_cache_spec_kind="full_attention")
    if kind == "BlockRemoved":
        return BlockRemoved(block_hashes=list(payload["block_hashes"]), medium=payload.get("medium"))
    if kind == "AllBlocksCleared":
        return AllBlocksCleared()
    raise ValueError(f"unknown KV event kind {kind!r}")

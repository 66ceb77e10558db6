"""kvd wire protocol: 4-byte big-endian length prefix + a msgpack map whose
``op`` field names the message.

The op codes, message fields, retention classes and tier names are a
contract with the engines' KV connectors, kept from the reference's daemon
(``infera/kvd/wire.py:57-728``). Keys are 8-byte block hashes.
"""

from __future__ import annotations

import asyncio
import dataclasses
import enum
import struct
from dataclasses import dataclass, field

import msgpack

LENGTH_PREFIX_BYTES = 4
MAX_FRAME = 1 << 31


class OpCode(str, enum.Enum):
    HELLO = "hello"
    GET = "get"
    BATCH_GET = "batch_get"
    SET = "set"
    BATCH_SET = "batch_set"
    SET_RESERVE = "set_reserve"
    SET_COMMIT = "set_commit"
    SET_CANCEL = "set_cancel"
    PREFETCH_HINT = "prefetch_hint"
    EXISTS = "exists"
    LOOKUP_TIER = "lookup_tier"
    REGISTER_FILE_ENTRY = "register_file_entry"
    CLEAR = "clear"
    STATS = "stats"
    HELLO_ACK = "hello_ack"
    GET_RESPONSE = "get_response"
    GET_SHARED_RESPONSE = "get_shared_response"
    BATCH_GET_RESPONSE = "batch_get_response"
    BATCH_GET_SHARED_RESPONSE = "batch_get_shared_response"
    SET_ACK = "set_ack"
    BATCH_SET_ACK = "batch_set_ack"
    SET_RESERVE_RESPONSE = "set_reserve_response"
    SET_COMMIT_RESPONSE = "set_commit_response"
    SET_CANCEL_RESPONSE = "set_cancel_response"
    EXISTS_RESPONSE = "exists_response"
    LOOKUP_TIER_RESPONSE = "lookup_tier_response"
    REGISTER_FILE_ENTRY_ACK = "register_file_entry_ack"
    CLEAR_ACK = "clear_ack"
    STATS_RESPONSE = "stats_response"
    ERROR = "error"


RETENTION_NONE = "none"
RETENTION_EPHEMERAL = "ephemeral"
RETENTION_SHORT = "short"
RETENTION_LONG = "long"
RETENTION_PRIORITY = {RETENTION_NONE: 0, RETENTION_EPHEMERAL: 10, RETENTION_SHORT: 50, RETENTION_LONG: 100}

TIER_MISS = "miss"
TIER_RAM = "ram"
TIER_FILE = "file"


@dataclass(frozen=True)
class Hello:
    client_id: str
    protocol_version: int = 1
    prefers_shared_arena: bool = False


@dataclass(frozen=True)
class HelloAck:
    server_id: str
    protocol_version: int = 1
    shared_arena: tuple | None = None   # (arena_size, slot_size, server_pid); the fd follows via SCM_RIGHTS


@dataclass(frozen=True)
class Get:
    key: bytes
    model: str = ""
    compat_key: str = ""


@dataclass(frozen=True)
class GetResponse:
    value: bytes | None
    retention: str | None = None


@dataclass(frozen=True)
class GetSharedResponse:
    slot_offset: int
    size: int
    version: int
    retention: str | None = None


@dataclass(frozen=True)
class BatchGet:
    keys: list
    model: str = ""
    compat_key: str = ""


@dataclass(frozen=True)
class BatchGetResponse:
    values: list


@dataclass(frozen=True)
class BatchGetSharedResponse:
    entries: list   # per key: (slot_offset, size, version) or None


@dataclass(frozen=True)
class Set:
    key: bytes
    value: bytes
    retention: str = RETENTION_SHORT
    model: str = ""
    compat_key: str = ""
    metadata: dict = field(default_factory=dict)
    ttl_seconds: float | None = None


@dataclass(frozen=True)
class SetAck:
    ok: bool
    reason: str = ""


@dataclass(frozen=True)
class BatchSet:
    keys: list
    values: list
    retention: str = RETENTION_SHORT
    model: str = ""
    compat_key: str = ""
    ttl_seconds: float | None = None


@dataclass(frozen=True)
class BatchSetAck:
    ok: list


@dataclass(frozen=True)
class SetReserve:
    key: bytes
    size: int
    retention: str = RETENTION_SHORT
    model: str = ""
    compat_key: str = ""
    ttl_seconds: float | None = None


@dataclass(frozen=True)
class SetReserveResponse:
    ok: bool
    lease_token: int = 0
    slot_id: int = 0
    payload_offset: int = 0
    payload_max_size: int = 0
    reason: str = ""


@dataclass(frozen=True)
class SetCommit:
    lease_token: int
    size: int


@dataclass(frozen=True)
class SetCommitResponse:
    ok: bool
    reason: str = ""


@dataclass(frozen=True)
class SetCancel:
    lease_token: int


@dataclass(frozen=True)
class SetCancelResponse:
    ok: bool


@dataclass(frozen=True)
class PrefetchHint:
    keys: list
    model: str = ""
    compat_key: str = ""
    deadline_ms: int = 1000


@dataclass(frozen=True)
class Exists:
    keys: list
    model: str = ""
    compat_key: str = ""


@dataclass(frozen=True)
class ExistsResponse:
    present: list


@dataclass(frozen=True)
class LookupTier:
    key: bytes
    model: str = ""
    compat_key: str = ""


@dataclass(frozen=True)
class LookupTierResponse:
    tier: str
    path: str | None = None
    file_offset: int = 0
    size: int = 0
    version: int = 0
    retention: str | None = None


@dataclass(frozen=True)
class RegisterFileEntry:
    key: bytes
    path: str
    file_offset: int = 0
    size: int = 0
    version: int = 0
    retention: str = RETENTION_SHORT
    model: str = ""
    compat_key: str = ""


@dataclass(frozen=True)
class RegisterFileEntryAck:
    ok: bool = True


@dataclass(frozen=True)
class Clear:
    model: str = ""
    compat_key: str = ""


@dataclass(frozen=True)
class ClearAck:
    cleared_entries: int


@dataclass(frozen=True)
class Stats:
    pass


@dataclass(frozen=True)
class StatsResponse:
    entries: int
    host_bytes: int
    spillover_bytes: int
    long_bytes: int
    gets_total: int
    sets_total: int
    hits_total: int
    misses_total: int
    evictions_total: int


@dataclass(frozen=True)
class ErrorMessage:
    code: str
    message: str = ""


_OP_OF = {
    Hello: OpCode.HELLO, HelloAck: OpCode.HELLO_ACK, Get: OpCode.GET, GetResponse: OpCode.GET_RESPONSE,
    GetSharedResponse: OpCode.GET_SHARED_RESPONSE, BatchGet: OpCode.BATCH_GET,
    BatchGetResponse: OpCode.BATCH_GET_RESPONSE, BatchGetSharedResponse: OpCode.BATCH_GET_SHARED_RESPONSE,
    Set: OpCode.SET, SetAck: OpCode.SET_ACK, BatchSet: OpCode.BATCH_SET, BatchSetAck: OpCode.BATCH_SET_ACK,
    SetReserve: OpCode.SET_RESERVE, SetReserveResponse: OpCode.SET_RESERVE_RESPONSE, SetCommit: OpCode.SET_COMMIT,
    SetCommitResponse: OpCode.SET_COMMIT_RESPONSE, SetCancel: OpCode.SET_CANCEL,
    SetCancelResponse: OpCode.SET_CANCEL_RESPONSE, PrefetchHint: OpCode.PREFETCH_HINT, Exists: OpCode.EXISTS,
    ExistsResponse: OpCode.EXISTS_RESPONSE, LookupTier: OpCode.LOOKUP_TIER,
    LookupTierResponse: OpCode.LOOKUP_TIER_RESPONSE, RegisterFileEntry: OpCode.REGISTER_FILE_ENTRY,
    RegisterFileEntryAck: OpCode.REGISTER_FILE_ENTRY_ACK, Clear: OpCode.CLEAR, ClearAck: OpCode.CLEAR_ACK,
    Stats: OpCode.STATS, StatsResponse: OpCode.STATS_RESPONSE, ErrorMessage: OpCode.ERROR,
}
_CLS_OF = {op.value: cls for cls, op in _OP_OF.items()}


def op_of(msg) -> OpCode:
    return _OP_OF[type(msg)]


def encode(msg) -> bytes:
    payload = {"op": _OP_OF[type(msg)].value}
    for f in dataclasses.fields(msg):
        payload[f.name] = getattr(msg, f.name)
    body = msgpack.packb(payload, use_bin_type=True)
    return struct.pack(">I", len(body)) + body


def decode_body(body: bytes):
    obj = msgpack.unpackb(body, raw=False)
    if not isinstance(obj, dict) or "op" not in obj:
        raise ValueError("frame is not a kvd message")
    cls = _CLS_OF.get(obj.pop("op"))
    if cls is None:
        raise ValueError("unknown op")
    names = {f.name for f in dataclasses.fields(cls)}
    kw = {k: v for k, v in obj.items() if k in names}
    if isinstance(kw.get("shared_arena"), list):
        kw["shared_arena"] = tuple(kw["shared_arena"])
    if cls is BatchGetSharedResponse:
        kw["entries"] = [tuple(e) if isinstance(e, list) else e for e in kw.get("entries", [])]
    return cls(**kw)


async def read_frame(reader: asyncio.StreamReader):
    hdr = await reader.readexactly(LENGTH_PREFIX_BYTES)
    n = struct.unpack(">I", hdr)[0]
    if n > MAX_FRAME:
        raise ValueError("frame too large")
    return decode_body(await reader.readexactly(n))


async def write_frame(writer: asyncio.StreamWriter, msg) -> None:
    writer.write(encode(msg))
    await writer.drain()

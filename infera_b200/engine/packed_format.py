"""KV chunk blob, version 2 - the on-disk / in-tier format of KV pages.

    [u32 LE header_len][msgpack header][zero padding][payload]

Header fields: ``v`` (2), ``chunk_tokens``, ``block_size``, ``num_layers``,
``layer_names``, ``hidden_dim`` (KV elements per token per channel),
``dtype`` (bf16 / fp16 / fp8_e4m3 / fp32), ``cache_group_id``,
``num_kv_channels`` (2 = K and V, 1 = an MLA latent) and
``payload_byte_offset`` (absolute offset of the payload, 4 KiB-aligned by
:func:`pack_chunk` so direct-I/O readers land on aligned offsets; 0 means
right after the header). The payload is ``[C, L, T, H]`` in ``dtype``.

The field names and byte layout are a format contract shared with the
reference's KV connector (``infera/engine/vllm/packed_format.py:81-385``)
so tiers written by either side stay readable.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

import msgpack

VERSION = 2
DTYPE_BYTES = {"bf16": 2, "fp16": 2, "fp8_e4m3": 1, "fp32": 4}


class PackedFormatError(Exception):
    """A blob that cannot be parsed; callers treat it as a cache miss."""


@dataclass(frozen=True)
class ChunkHeader:
    chunk_tokens: int
    block_size: int
    num_layers: int
    hidden_dim: int
    dtype: str = "bf16"
    layer_names: tuple = ()
    cache_group_id: int = 0
    num_kv_channels: int = 2
    payload_byte_offset: int = 0
    version: int = VERSION

    @property
    def payload_bytes(self) -> int:
        return self.num_kv_channels * self.num_layers * self.chunk_tokens * self.hidden_dim * DTYPE_BYTES[self.dtype]


def _header_body(h: ChunkHeader) -> bytes:
    return msgpack.packb({
        "v": VERSION, "chunk_tokens": int(h.chunk_tokens), "block_size": int(h.block_size),
        "num_layers": int(h.num_layers), "layer_names": list(h.layer_names), "hidden_dim": int(h.hidden_dim),
        "dtype": str(h.dtype), "cache_group_id": int(h.cache_group_id), "num_kv_channels": int(h.num_kv_channels),
        "payload_byte_offset": int(h.payload_byte_offset)}, use_bin_type=True)


def pack_header(h: ChunkHeader, align: int = 4096) -> tuple[bytes, ChunkHeader]:
    """Header bytes padded so the payload starts at a multiple of ``align``."""
    body = _header_body(h)
    # the offset is part of the header, so iterate until it is stable
    off = 0
    for _ in range(3):
        h = ChunkHeader(**{**h.__dict__, "payload_byte_offset": off})
        body = _header_body(h)
        need = 4 + len(body)
        off_new = (need + align - 1) // align * align if align else need
        if off_new == off:
            break
        off = off_new
    h = ChunkHeader(**{**h.__dict__, "payload_byte_offset": off})
    body = _header_body(h)
    raw = struct.pack("<I", len(body)) + body
    return raw + b"\0" * (off - len(raw)), h


def pack_chunk(h: ChunkHeader, payload, align: int = 4096) -> bytearray:
    """Header + payload in one buffer (the payload is copied once)."""
    hdr, h = pack_header(h, align)
    n = memoryview(payload).nbytes
    if n != h.payload_bytes:
        raise PackedFormatError(f"payload is {n} bytes, header says {h.payload_bytes}")
    out = bytearray(len(hdr) + n)
    out[:len(hdr)] = hdr
    out[len(hdr):] = memoryview(payload).cast("B")
    return out


def unpack_header(blob) -> ChunkHeader:
    if len(blob) < 4:
        raise PackedFormatError("blob shorter than its length prefix")
    n = struct.unpack_from("<I", blob, 0)[0]
    if 4 + n > len(blob):
        raise PackedFormatError("truncated header")
    try:
        d = msgpack.unpackb(bytes(blob[4:4 + n]), raw=False)
    except Exception as e:
        raise PackedFormatError(f"bad header: {e}") from e
    if d.get("v") != VERSION:
        raise PackedFormatError(f"unsupported chunk version {d.get('v')}")
    h = ChunkHeader(chunk_tokens=d["chunk_tokens"], block_size=d["block_size"], num_layers=d["num_layers"],
                    hidden_dim=d["hidden_dim"], dtype=d["dtype"], layer_names=tuple(d.get("layer_names") or ()),
                    cache_group_id=d.get("cache_group_id", 0), num_kv_channels=d.get("num_kv_channels", 2),
                    payload_byte_offset=d.get("payload_byte_offset", 0) or 4 + n)
    if h.dtype not in DTYPE_BYTES:
        raise PackedFormatError(f"unknown dtype {h.dtype}")
    return h


def unpack_chunk(blob) -> tuple[ChunkHeader, memoryview]:
    h = unpack_header(blob)
    off = h.payload_byte_offset
    if off + h.payload_bytes > len(blob):
        raise PackedFormatError("truncated payload")
    return h, memoryview(blob)[off: off + h.payload_bytes]

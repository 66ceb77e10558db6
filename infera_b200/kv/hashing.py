"""Block hashing of the tier-aware KV index.

    seed           = 1337 XOR lora_hash (0 without an adapter)
    block_hash_i   = XXH3_64(tokens of block i as u32 LE, seed)
                     (media spans overlapping the block mix in
                      u64 LE media_hash || u32 LE start-in-block || u32 LE length)
    sequence_hash_i = XXH3_64(sequence_hash_{i-1} u64 LE || block_hash_i u64 LE, seed),
                     sequence_hash_{-1} = 0

A trailing partial block is not hashed. This is the index's own scheme
(seeded apart from the router's seed-0 chain so the two can never be
confused); the reference's index uses a seed-1337 chain of the same shape
(``infera/kv/hashing.py:38-215``).
"""

from __future__ import annotations

import struct

import numpy as np
import xxhash

from infera_b200.kv.types import BlockKey, MmRun

BASE_SEED = 1337
MASK64 = (1 << 64) - 1


def seed_for(lora_hash: int = 0) -> int:
    return (BASE_SEED ^ (lora_hash & MASK64)) & MASK64


def lora_hash(name: str | None) -> int:
    return 0 if not name else xxhash.xxh3_64_intdigest(name.encode())


def hash_token_blocks(tokens, block_size: int, lora: int = 0, mm_runs: list[MmRun] | None = None,
                      parent_sequence_hash: int = 0) -> list[BlockKey]:
    seed = seed_for(lora)
    arr = np.asarray(tokens, dtype=np.uint32)
    n = len(arr) // block_size
    out: list[BlockKey] = []
    seq = parent_sequence_hash
    for i in range(n):
        lo, hi = i * block_size, (i + 1) * block_size
        buf = arr[lo:hi].tobytes()
        for r in mm_runs or ():
            if r.start < hi and r.start + r.length > lo:
                buf += struct.pack("<QII", r.media_hash & MASK64, max(0, r.start - lo), r.length)
        bh = xxhash.xxh3_64_intdigest(buf, seed=seed)
        seq = xxhash.xxh3_64_intdigest(struct.pack("<QQ", seq, bh), seed=seed)
        out.append(BlockKey(bh, seq))
    return out


def hash_prompt(tokens, block_size: int, lora_name: str | None = None, mm_runs=None) -> list[BlockKey]:
    return hash_token_blocks(tokens, block_size, lora_hash(lora_name), mm_runs)

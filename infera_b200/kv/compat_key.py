"""Compatibility key: two publishers' cached blocks are interchangeable only
if everything that shapes the KV bytes matches - model family and name,
tokenizer (digest, plus the ids of a canary string as a runtime check),
index block size, KV dtype, and attention role (prefill / decode pools of
one model keep separate trees). Role of ``infera/kv/compat_key.py:128``.
"""

from __future__ import annotations

import hashlib
import json

from infera_b200.kv.families import family_of
from infera_b200.utils.tokenizer import CANARY_STRING


def compat_key(model_name: str, tokenizer_digest: str, block_size: int, kv_dtype: str = "bf16",
               role: str = "mixed", extra: dict | None = None) -> str:
    body = {"family": family_of(model_name), "model": model_name, "tokenizer": tokenizer_digest,
            "block_size": int(block_size), "kv_dtype": kv_dtype, "role": role, **(extra or {})}
    return hashlib.sha256(json.dumps(body, sort_keys=True).encode()).hexdigest()[:24]


def canary_ids(tokenizer) -> list[int]:
    return list(tokenizer.encode(CANARY_STRING))

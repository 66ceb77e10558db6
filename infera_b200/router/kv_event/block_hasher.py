"""Request body -> chained router block hashes.

Tokenizes with the same tokenizer as the engine
(:func:`infera_b200.utils.tokenizer.request_token_ids`), caches the ids on
the body, then hashes full blocks (``infera/router/kv_event/block_hasher.py``
does the same for vLLM / SGLang tokenizers)."""

from __future__ import annotations

from infera_b200.utils.hashing import chain_hashes
from infera_b200.utils.tokenizer import load_tokenizer, request_token_ids


class BlockHasher:
    def __init__(self, tokenizer=None):
        self.tok = tokenizer or load_tokenizer(None)

    def token_ids(self, request: dict) -> list[int]:
        ids = request.get("_infera_token_ids")
        if not isinstance(ids, list):
            try:
                ids = request_token_ids(request, self.tok)
            except Exception:
                ids = []
            request["_infera_token_ids"] = ids
        return ids

    def hash_for(self, request: dict, block_size: int, engine=None) -> list[int]:
        cache = request.setdefault("_infera_hash_cache", {})
        if block_size in cache:
            return cache[block_size]
        hs = chain_hashes(self.token_ids(request), block_size)
        cache[block_size] = hs
        return hs

"""Client cache hints: Anthropic ``cache_control`` blocks and OpenAI
``prompt_cache_key`` / ``prompt_cache_retention``.

Behaviour follows ``infera/router/cache_control.py:67-466``:

* retention levels none < short < long; the strongest hint in a body wins;
* Anthropic ``{"type": "ephemeral"}`` -> short, ``"ttl": "1h"`` -> long;
  ``thinking`` / ``redacted_thinking`` blocks never cache;
* OpenAI ``prompt_cache_retention`` "24h"/"1h"/"long" -> long,
  "5m"/"short" -> short, "none"/"off"/"disabled" -> none; a bare
  ``prompt_cache_key`` is an implicit short hint;
* any image / audio / video / file content marks the body multimodal (the
  router then ignores token-prefix locality, whose hashes cannot see the
  media), and each media reference gets a stable key (XXH3-64 of the URL or
  data URI) for image affinity;
* requests with no hint are treated as ``INFERA_ROUTER_DEFAULT_RETENTION``
  (default long) by :func:`effective_retention`.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from enum import Enum
from typing import Any, Iterator

from xxhash import xxh3_64_intdigest


class Retention(str, Enum):
    NONE = "none"
    SHORT = "short"
    LONG = "long"

    def rank(self) -> int:
        return _RANK[self.value]


_RANK = {"none": 0, "short": 1, "long": 2}


@dataclass(frozen=True)
class CacheHints:
    retention: Retention
    session_id: str | None
    explicit_hint_seen: bool
    has_multimodal_content: bool = False


MM_BLOCK_TYPES = frozenset({"image", "image_url", "input_image", "audio", "input_audio", "video", "video_url",
                            "file", "input_file", "document"})
_NO_CACHE_TYPES = frozenset({"thinking", "redacted_thinking"})


def _default_retention() -> Retention:
    try:
        return Retention(os.environ.get("INFERA_ROUTER_DEFAULT_RETENTION", "long").strip().lower())
    except ValueError:
        return Retention.LONG


def effective_retention(r: Retention) -> Retention:
    return r if r != Retention.NONE else _default_retention()


def _openai_retention(body: dict) -> Retention | None:
    v = body.get("prompt_cache_retention")
    if isinstance(v, str):
        v = v.strip().lower()
        if v in ("24h", "1h", "long"):
            return Retention.LONG
        if v in ("5m", "short"):
            return Retention.SHORT
        if v in ("none", "off", "disabled"):
            return Retention.NONE
        return None
    if body.get("prompt_cache_key"):
        return Retention.SHORT
    return None


def _blocks_with_cache_control(body: dict) -> Iterator[dict]:
    system = body.get("system")
    if isinstance(system, list):
        yield from (b for b in system if isinstance(b, dict) and "cache_control" in b)
    tools = body.get("tools")
    if isinstance(tools, list):
        yield from (t for t in tools if isinstance(t, dict) and "cache_control" in t)
    for msg in body.get("messages") or []:
        if isinstance(msg, dict) and isinstance(msg.get("content"), list):
            yield from (b for b in msg["content"] if isinstance(b, dict) and "cache_control" in b)


def _block_retention(block: dict) -> Retention | None:
    if block.get("type") in _NO_CACHE_TYPES:
        return Retention.NONE
    cc = block.get("cache_control")
    if not isinstance(cc, dict):
        return None
    if cc.get("type") != "ephemeral":
        return None
    ttl = cc.get("ttl")
    if isinstance(ttl, str) and ttl.strip().lower() in ("1h", "60m", "3600s"):
        return Retention.LONG
    return Retention.SHORT


def _iter_content_blocks(body: dict) -> Iterator[dict]:
    for msg in body.get("messages") or []:
        if isinstance(msg, dict) and isinstance(msg.get("content"), list):
            yield from (b for b in msg["content"] if isinstance(b, dict))
    system = body.get("system")
    if isinstance(system, list):
        yield from (b for b in system if isinstance(b, dict))


def detect_multimodal(body: dict) -> bool:
    for b in _iter_content_blocks(body):
        t = b.get("type")
        if isinstance(t, str) and t in MM_BLOCK_TYPES:
            return True
    if isinstance(body.get("images"), list) and body["images"]:
        return True
    if isinstance(body.get("audio"), (dict, list)) and body["audio"]:
        return True
    return False


def _media_ref(block: dict) -> str | None:
    iu = block.get("image_url")
    if isinstance(iu, str):
        return iu
    if isinstance(iu, dict) and isinstance(iu.get("url"), str):
        return iu["url"]
    ia = block.get("input_audio")
    if isinstance(ia, dict) and isinstance(ia.get("data"), str):
        return ia["data"]
    src = block.get("source")
    if isinstance(src, dict):
        for k in ("url", "data"):
            if isinstance(src.get(k), str):
                return src[k]
    for k in ("url", "data"):
        if isinstance(block.get(k), str):
            return block[k]
    return None


def extract_image_keys(body: Any) -> list[int]:
    """XXH3-64 of each media reference in document order."""
    keys: list[int] = []
    if not isinstance(body, dict):
        return keys

    def push(ref):
        if isinstance(ref, str) and ref.strip():
            keys.append(xxh3_64_intdigest(ref.strip().encode("utf-8")))

    for b in _iter_content_blocks(body):
        push(_media_ref(b))
    for im in body.get("images") or []:
        push(im if isinstance(im, str) else (_media_ref(im) if isinstance(im, dict) else None))
    return keys


def parse_cache_hints(body: Any) -> CacheHints:
    if not isinstance(body, dict):
        return CacheHints(Retention.NONE, None, False, False)
    oa = _openai_retention(body)
    sess = body.get("prompt_cache_key") or body.get("session_id")
    sess = sess.strip() if isinstance(sess, str) and sess.strip() else None
    found = [r for r in (_block_retention(b) for b in _blocks_with_cache_control(body)) if r is not None]
    an = max(found, key=Retention.rank) if found else None
    mm = detect_multimodal(body)
    cands = [r for r in (oa, an) if r is not None]
    if not cands:
        return CacheHints(Retention.NONE, sess, False, mm)
    return CacheHints(max(cands, key=Retention.rank), sess, bool(found) or oa is not None, mm)

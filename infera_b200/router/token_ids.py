"""Generated-token bookkeeping carried in worker responses.

Workers asked with ``return_token_ids`` put ``token_ids`` on each choice
(and ``prompt_token_ids`` on the first); the router reads them for migration
and strips them before the client sees the chunk
(``infera/router/token_ids.py:33-134`` handles vLLM's and SGLang's shapes;
both are read here)."""

from __future__ import annotations

import json


def parse_sse_json(ev: bytes) -> dict | None:
    line = ev.strip()
    if not line.startswith(b"data:"):
        return None
    payload = line[5:].strip()
    if payload == b"[DONE]" or not payload:
        return None
    try:
        return json.loads(payload)
    except ValueError:
        return None


def choice_token_ids(obj: dict) -> list[int]:
    out: list[int] = []
    for ch in obj.get("choices") or []:
        ids = ch.get("token_ids")
        if ids is None:
            ext = (ch.get("sglext") or obj.get("sglext") or {})
            ids = ext.get("output_ids")
        if isinstance(ids, list):
            out.extend(int(x) for x in ids)
    return out


def choice_text(obj: dict) -> str:
    parts = []
    for ch in obj.get("choices") or []:
        if "text" in ch and isinstance(ch["text"], str):
            parts.append(ch["text"])
        delta = ch.get("delta") or {}
        if isinstance(delta.get("content"), str):
            parts.append(delta["content"])
    return "".join(parts)


def finish_reason(obj: dict) -> str | None:
    for ch in obj.get("choices") or []:
        if ch.get("finish_reason"):
            return ch["finish_reason"]
    return None


def strip_token_ids(obj: dict) -> dict:
    obj.pop("prompt_token_ids", None)
    obj.pop("sglext", None)
    for ch in obj.get("choices") or []:
        ch.pop("token_ids", None)
        ch.pop("prompt_token_ids", None)
        ch.pop("sglext", None)
    return obj


def to_sse(obj: dict) -> bytes:
    return b"data: " + json.dumps(obj, separators=(",", ":")).encode() + b"\n\n"

"""Canonical model-family names for compatibility keys: checkpoints of one
family with one tokenizer can share cached KV only if every other part of
the key also matches (role of ``infera/kv/families.py:13-144``)."""

from __future__ import annotations

import re

_RULES: list[tuple[str, str]] = [
    (r"deepseek[-_]?v3|deepseek[-_]?r1", "deepseek-v3"),
    (r"deepseek[-_]?v2", "deepseek-v2"),
    (r"kimi[-_]?k2", "kimi-k2"),
    (r"llama[-_]?3", "llama-3"),
    (r"llama[-_]?2", "llama-2"),
    (r"qwen[-_]?3", "qwen3"),
    (r"qwen[-_]?2", "qwen2"),
    (r"glm[-_]?4|glm[-_]?5", "glm"),
    (r"mistral|mixtral", "mistral"),
    (r"gpt[-_]?oss", "gpt-oss"),
]


def family_of(model_name: str) -> str:
    m = model_name.lower().rsplit("/", 1)[-1]
    for pat, fam in _RULES:
        if re.search(pat, m):
            return fam
    return re.sub(r"[^a-z0-9]+", "-", m).strip("-") or "unknown"

"""Redaction of credentials before strings reach logs or error bodies.

Bearer tokens, API keys in URLs / headers / JSON and passwords in DSNs are
replaced by ``***`` (role of ``infera/common/logsafe.py:20``)."""

from __future__ import annotations

import re

_PATTERNS = [
    (re.compile(r"(?i)(bearer\s+)[A-Za-z0-9._~+/=-]{8,}"), r"\1***"),
    (re.compile(r"(?i)((?:api[_-]?key|token|secret|password|passwd|authorization)[\"']?\s*[:=]\s*[\"']?)"
                r"[^\s\"',&]{4,}"), r"\1***"),
    (re.compile(r"(?i)([?&](?:api[_-]?key|token|access_token|sig|signature)=)[^&\s]+"), r"\1***"),
    (re.compile(r"(://[^:/@\s]+:)[^@/\s]+(@)"), r"\1***\2"),
    (re.compile(r"\b(sk|hf|ghp|gho|xox[bap])[-_][A-Za-z0-9_-]{12,}\b"), r"\1-***"),
]


def scrub(text) -> str:
    s = str(text)
    for pat, rep in _PATTERNS:
        s = pat.sub(rep, s)
    return s

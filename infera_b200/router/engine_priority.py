"""Carry the client's retention hint to the engine.

This framework's engine reads ``kv_transfer_params.infera_retention``
(and ``priority`` for SGLang-style engines), which orders prefix-cache
eviction and tier spills (``infera/router/engine_priority.py:58-110``)."""

from __future__ import annotations

from infera_b200.router.cache_control import CacheHints, effective_retention

SGLANG_PRIORITY = {"none": 0, "short": 50, "long": 100}


def inject_engine_priority(body: dict, hints: CacheHints | None, engine) -> dict:
    if hints is None:
        return body
    out = dict(body)
    ret = effective_retention(hints.retention).value
    eng = getattr(engine, "value", str(engine))
    if eng == "sglang":
        out.setdefault("priority", SGLANG_PRIORITY[ret])
        out["infera_retention"] = ret
    else:
        ktp = dict(out.get("kv_transfer_params") or {})
        ktp.setdefault("infera_retention", ret)
        out["kv_transfer_params"] = ktp
    return out

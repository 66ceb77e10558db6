"""Reading an engine's Prometheus exposition: how much work is in flight.

Drain and scaling decisions ask one question of a worker's ``/metrics``:
how many requests has it accepted and not finished? Each engine spells the
gauges differently, exposes one series per rank (which must be summed: a
busy rank must not hide behind an idle one), and a missing series means
"unknown", never "idle". PD handoff queues count as in flight while
draining (a prefill worker can look idle while its KV is still moving).
Names and semantics follow ``infera/common/engine_metrics.py:47-162``.
"""

from __future__ import annotations

import re

from infera_b200.common.worker_pool import EngineType

# key -> engine -> spellings, newest first
NAMES: dict[str, dict[EngineType, tuple[str, ...]]] = {
    "requests_running": {
        EngineType.INFERA_B200: ("infera_engine:num_requests_running",),
        EngineType.VLLM: ("vllm:num_requests_running",),
        EngineType.SGLANG: ("sglang:num_running_reqs",),
    },
    "requests_waiting": {
        EngineType.INFERA_B200: ("infera_engine:num_requests_waiting",),
        EngineType.VLLM: ("vllm:num_requests_waiting",),
        EngineType.SGLANG: ("sglang:num_queue_reqs",),
    },
    "kv_cache_usage": {
        EngineType.INFERA_B200: ("infera_engine:kv_cache_usage_perc",),
        EngineType.VLLM: ("vllm:kv_cache_usage_perc", "vllm:gpu_cache_usage_perc"),
        EngineType.SGLANG: ("sglang:token_usage",),
    },
}

# gauges that are unfinished work only from a drain's point of view
DRAIN_EXTRA: dict[EngineType, tuple[str, ...]] = {
    EngineType.INFERA_B200: ("infera_engine:pd_push_queue",),
    EngineType.SGLANG: ("sglang:num_prefill_bootstrap_queue_reqs", "sglang:num_prefill_inflight_queue_reqs",
                        "sglang:num_decode_prealloc_queue_reqs", "sglang:num_decode_transfer_queue_reqs"),
}

_SAMPLE = re.compile(r"^(?P<name>[A-Za-z_:][A-Za-z0-9_:]*)(?:\{[^}]*\})?\s+(?P<value>[-+0-9.eEinfNa]+)(?:\s+\d+)?\s*$")


def parse_exposition(text: str) -> dict[str, float]:
    """Sum of every series of each metric name (labels collapsed)."""
    out: dict[str, float] = {}
    for line in text.splitlines():
        if not line or line[0] == "#":
            continue
        m = _SAMPLE.match(line.strip())
        if not m:
            continue
        try:
            v = float(m.group("value"))
        except ValueError:
            continue
        out[m.group("name")] = out.get(m.group("name"), 0.0) + v
    return out


def parse_metric(text: str, name: str) -> float | None:
    return parse_exposition(text).get(name)


def _engine(engine) -> EngineType:
    return engine if isinstance(engine, EngineType) else EngineType(str(engine))


def read_gauge(text: str, key: str, engine) -> float | None:
    """First spelling of ``key`` the exposition has (None if none)."""
    vals = parse_exposition(text)
    for name in NAMES[key].get(_engine(engine), ()):
        if name in vals:
            return vals[name]
    return None


def inflight_from_metrics(text: str, engine, draining: bool = True) -> float | None:
    """running + waiting (+ PD handoff queues when draining); None = unknown."""
    eng = _engine(engine)
    vals = parse_exposition(text)
    run = next((vals[n] for n in NAMES["requests_running"].get(eng, ()) if n in vals), None)
    wait = next((vals[n] for n in NAMES["requests_waiting"].get(eng, ()) if n in vals), None)
    if run is None or wait is None:
        return None
    total = run + wait
    if draining:
        total += sum(vals.get(n, 0.0) for n in DRAIN_EXTRA.get(eng, ()))
    return total

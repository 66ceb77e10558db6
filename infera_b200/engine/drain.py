"""Drain an engine reached only through its HTTP ``/metrics``.

For engines that do not report in-flight work exactly (external engines
behind this fleet's launcher), the drain polls ``/metrics`` until the
in-flight count (running + waiting + PD handoff queues) has stayed at 0 for
a settle window, bounded by a timeout. An engine whose metrics cannot be
read, or whose in-flight gauge is missing, is not waited on (unknown is
not idle, but waiting forever on it would block shutdown). This
framework's own engine reports in-flight exactly and drains without a
settle window. Behaviour of ``infera/engine/drain.py:61-140``.
"""

from __future__ import annotations

import asyncio
import logging
import time

from infera_b200.common.engine_metrics import inflight_from_metrics

logger = logging.getLogger(__name__)

SETTLE_S = 6.0


async def drain_engine_inflight(fetch_metrics, engine, timeout: float = 30.0, settle_s: float = SETTLE_S,
                                poll_s: float = 0.5, clock=time.monotonic, sleep=asyncio.sleep) -> dict:
    """``fetch_metrics()``: async, returns the exposition text.

    Returns {"drained": bool, "reason": str, "waited_s": float}."""
    t0 = clock()
    idle_since = None
    while True:
        try:
            text = await fetch_metrics()
        except Exception as e:
            logger.warning("drain: metrics unreadable (%s); not waiting", e)
            return {"drained": False, "reason": "metrics_unreadable", "waited_s": clock() - t0}
        n = inflight_from_metrics(text, engine, draining=True)
        if n is None:
            return {"drained": False, "reason": "inflight_unknown", "waited_s": clock() - t0}
        now = clock()
        if n <= 0:
            idle_since = idle_since if idle_since is not None else now
            if now - idle_since >= settle_s:
                return {"drained": True, "reason": "idle", "waited_s": now - t0}
        else:
            idle_since = None
        if now - t0 >= timeout:
            return {"drained": False, "reason": "timeout", "waited_s": now - t0}
        await sleep(poll_s)

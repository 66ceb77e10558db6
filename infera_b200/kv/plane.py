"""The router's tier-aware KV index data plane, assembled.

One :class:`~infera_b200.kv.index.KVIndex`, its single writer, a ZMQ
subscriber per publishing worker and the 30 s snapshot reconciler, driven
by the registry: a worker whose registration carries a ``kv`` block with
``supports_events`` and an ``events_endpoint`` is subscribed and becomes a
reconciliation target (snapshots from ``{snapshot_endpoint}/v1/kv-snapshot
?model=&compat_key=``); one that leaves is unsubscribed and its trees are
dropped. Role of the Phase-1 block of ``infera/server/__main__.py:66-190``.
"""

from __future__ import annotations

import asyncio
import logging

from infera_b200.kv.index import KVIndex
from infera_b200.kv.writer import KvIndexSubscriber, KvIndexWriter, SnapshotReconciler

logger = logging.getLogger(__name__)


def http_snapshot_fetch(timeout: float = 10.0):
    """``fetch(target)`` for the reconciler: GET the publisher's snapshot."""
    import httpx

    async def fetch(target):
        url, model, compat = target[0], target[1], target[2]
        async with httpx.AsyncClient(timeout=timeout) as c:
            r = await c.get(url.rstrip("/") + "/v1/kv-snapshot", params={"model": model, "compat_key": compat})
            r.raise_for_status()
            return r.json()

    return fetch


class KvIndexPlane:
    def __init__(self, fetch=None, period_s: float = 30.0):
        self.index = KVIndex()
        self.writer = KvIndexWriter(self.index)
        self.subscribers = KvIndexSubscriber(self.writer)
        # worker id -> (snapshot url, model, compat key, events endpoint)
        self.targets: dict[str, tuple[str, str, str, str]] = {}
        self.reconciler = SnapshotReconciler(self.index, lambda: list(self.targets.values()),
                                             fetch or http_snapshot_fetch(), period_s)
        self._loop: asyncio.AbstractEventLoop | None = None
        self._task: asyncio.Task | None = None

    async def start(self) -> None:
        self._loop = asyncio.get_running_loop()
        self.writer.start()
        self._task = self._loop.create_task(self.reconciler.run())
        for t in self.targets.values():     # workers seen before the loop ran
            self.subscribers.add(t[3])

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass
        await self.subscribers.stop()
        await self.writer.stop()

    def _in_loop(self, fn, *a) -> None:
        if self._loop is None:
            return
        try:
            running = asyncio.get_running_loop()
        except RuntimeError:
            running = None
        if running is self._loop:
            fn(*a)
        else:
            self._loop.call_soon_threadsafe(fn, *a)

    def on_worker_added(self, w) -> None:
        kv = getattr(w, "kv", None)
        if kv is None or not kv.supports_events or not kv.events_endpoint:
            return
        t = (kv.snapshot_endpoint or w.url, w.model_name, kv.tokenizer_digest, kv.events_endpoint)
        self.targets[w.worker_id] = t
        logger.info("kv-index: subscribing to %s at %s", w.worker_id, kv.events_endpoint)
        self._in_loop(self.subscribers.add, kv.events_endpoint)

    def on_worker_removed(self, w) -> None:
        wid = getattr(w, "worker_id", w)
        t = self.targets.pop(wid, None)
        if t is not None:
            self._in_loop(self.subscribers.remove, t[3])
        self._in_loop(self.index.drop_publisher, wid)

    def stats(self) -> dict:
        s = self.index.size()
        return {
            "index": {"trees": s.trees, "nodes": s.nodes, "optimistic": s.optimistic,
                      "stored_events": s.stored_events, "removed_events": s.removed_events,
                      "dropped_unknown_parent": s.dropped_unknown_parent},
            "writer": {"batches_applied": self.writer.applied, "batches_dropped_overload": self.writer.dropped},
            "subscribers": {"endpoints": sorted(t[3] for t in self.targets.values()),
                            "batches_dropped_malformed": self.subscribers.decode_errors},
            "reconciler": {"rounds": self.reconciler.rounds, "snapshots_failed": self.reconciler.failures},
        }

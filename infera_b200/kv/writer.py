"""Single writer of the KV index, its ZMQ subscriber pool and the
snapshot reconciler.

``KvIndexWriter`` drains an asyncio queue of ``EventBatch`` es and applies
them to the index in order (one writer: no locks on the tree; readers run
on the same loop between batches). ``KvIndexSubscriber`` feeds that queue
from one ZMQ SUB socket per publisher endpoint (reconnecting with backoff).
``SnapshotReconciler`` periodically (30 s) fetches each publisher's
snapshot and resets its tree to it, repairing anything a lost event left
wrong. Roles of ``infera/kv/writer.py:42``, ``infera/kv/subscriber.py:47-162``
and ``infera/kv/snapshot.py:205``.
"""

from __future__ import annotations

import asyncio
import logging

from infera_b200.kv.index import KVIndex
from infera_b200.kv.wire import TOPIC, EventBatch, decode_batch, snapshot_chains

logger = logging.getLogger(__name__)


class KvIndexWriter:
    def __init__(self, index: KVIndex, maxsize: int = 65536):
        self.index = index
        self.queue: asyncio.Queue = asyncio.Queue(maxsize=maxsize)
        self.applied = 0
        self.dropped = 0
        self._task: asyncio.Task | None = None

    def submit(self, batch: EventBatch) -> bool:
        try:
            self.queue.put_nowait(batch)
            return True
        except asyncio.QueueFull:
            self.dropped += 1
            return False

    def apply(self, b: EventBatch) -> None:
        key = (b.model, b.compat, b.publisher)
        for e in b.events:
            if e.kind == "stored":
                self.index.apply_stored(key, e.blocks, e.parent, e.tier)
            elif e.kind == "removed":
                self.index.apply_removed(key, e.removed, e.tier)
            elif e.kind == "cleared":
                self.index.clear(key, e.tier)
        self.applied += 1

    async def run(self) -> None:
        while True:
            b = await self.queue.get()
            try:
                self.apply(b)
            except Exception:
                logger.exception("applying a kv-index batch failed")

    def start(self) -> None:
        self._task = asyncio.get_running_loop().create_task(self.run())

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass


class KvIndexSubscriber:
    def __init__(self, writer: KvIndexWriter):
        self.writer = writer
        self._tasks: dict[str, asyncio.Task] = {}
        self.decode_errors = 0

    def add(self, endpoint: str) -> None:
        if endpoint not in self._tasks:
            self._tasks[endpoint] = asyncio.get_running_loop().create_task(self._sub(endpoint))

    def remove(self, endpoint: str) -> None:
        t = self._tasks.pop(endpoint, None)
        if t is not None:
            t.cancel()

    async def _sub(self, endpoint: str) -> None:
        import zmq
        import zmq.asyncio

        ctx = zmq.asyncio.Context.instance()
        backoff = 0.25
        while True:
            sock = ctx.socket(zmq.SUB)
            try:
                sock.connect(endpoint)
                sock.subscribe(TOPIC)
                while True:
                    frames = await sock.recv_multipart()
                    try:
                        self.writer.submit(decode_batch(frames[-1]))
                    except Exception:
                        self.decode_errors += 1
                backoff = 0.25
            except asyncio.CancelledError:
                raise
            except Exception as e:
                logger.warning("kv-index subscriber %s failed (%s)", endpoint, e)
                await asyncio.sleep(backoff)
                backoff = min(5.0, backoff * 2)
            finally:
                sock.close(linger=0)

    async def stop(self) -> None:
        for t in self._tasks.values():
            t.cancel()
        self._tasks.clear()


class SnapshotReconciler:
    """``fetch(target) -> snapshot dict``; ``publishers() -> [target]`` (a
    target is whatever ``fetch`` understands: a URL, or a tuple)."""

    def __init__(self, index: KVIndex, publishers, fetch, period_s: float = 30.0):
        self.index = index
        self.publishers = publishers
        self.fetch = fetch
        self.period_s = period_s
        self.rounds = 0
        self.failures = 0

    async def reconcile_once(self) -> int:
        n = 0
        for url in self.publishers():
            try:
                snap = await self.fetch(url)
            except Exception as e:
                self.failures += 1
                logger.warning("kv-index snapshot from %s failed: %s", url, e)
                continue
            self.index.replace((snap["model"], snap["compat"], snap["publisher"]), snapshot_chains(snap))
            n += 1
        self.rounds += 1
        return n

    async def run(self) -> None:
        while True:
            await asyncio.sleep(self.period_s)
            await self.reconcile_once()

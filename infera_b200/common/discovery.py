"""Fleet discovery: keeps a :class:`WorkerPool` in sync with the workers'
registration records.

* :class:`EtcdRegistry` - etcd v3 over its HTTP/JSON gateway: one range read
  of the prefix, then a streaming watch from the next revision; PUT ->
  upsert, DELETE -> remove; reconnects with backoff and re-reads on a broken
  stream (behaviour of ``infera/common/discovery.py:100-330``).
* :class:`InProcessRegistry` - the same callbacks for workers living in the
  same process (tests, the CPU fleet harness, single-process deployments).

Both verify the tokenizer canary of records that carry a ``kv`` block and
fan ``on_worker_added`` / ``on_worker_removed`` out to listeners (the
policy's event subscriptions, the cache-view reconciler).
"""

from __future__ import annotations

import asyncio
import base64
import json
import logging
from typing import Callable

import httpx

from infera_b200.common.worker_pool import (CanaryMismatch, CanaryVerifier, WorkerInfo, WorkerPool, WorkerStatus,
                                            worker_info_from_json)

logger = logging.getLogger(__name__)

DEFAULT_PREFIX = "/infera/workers/"
Listener = Callable[[WorkerInfo], None]


def normalize_endpoint(endpoint: str) -> str:
    if endpoint.startswith(("http://", "https://")):
        return endpoint.rstrip("/")
    if ":" not in endpoint:
        endpoint += ":2379"
    return "http://" + endpoint


def b64(s: str | bytes) -> str:
    if isinstance(s, str):
        s = s.encode()
    return base64.b64encode(s).decode()


def unb64(s: str) -> bytes:
    return base64.b64decode(s)


def prefix_range_end(prefix: str) -> bytes:
    pb = prefix.encode()
    if not pb:
        return b"\x00"
    return pb[:-1] + bytes([pb[-1] + 1])


class _RegistryBase:
    def __init__(self, pool: WorkerPool | None = None) -> None:
        self.pool = pool or WorkerPool()
        self.canary = CanaryVerifier()
        self._added: list[Listener] = []
        self._removed: list[Listener] = []
        self.rejected: dict[str, str] = {}

    def on_worker_added(self, fn: Listener) -> None:
        self._added.append(fn)

    def on_worker_removed(self, fn: Listener) -> None:
        self._removed.append(fn)

    def _upsert(self, w: WorkerInfo) -> bool:
        if w.kv is not None:
            try:
                self.canary.verify(model_name=w.model_name, worker_id=w.worker_id, canary=w.kv.tokenizer_canary)
            except CanaryMismatch as e:
                logger.error("rejecting worker: %s", e)
                self.rejected[w.worker_id] = str(e)
                return False
        existed = self.pool.get(w.worker_id) is not None
        self.pool.add(w)
        if not existed:
            for fn in self._added:
                try:
                    fn(w)
                except Exception:  # listeners must not break discovery
                    logger.exception("on_worker_added listener failed")
        return True

    def _remove(self, worker_id: str) -> None:
        w = self.pool.remove(worker_id)
        if w is None:
            return
        if not any(x.model_name == w.model_name for x in self.pool.all()):
            self.canary.forget(w.model_name)
        for fn in self._removed:
            try:
                fn(w)
            except Exception:
                logger.exception("on_worker_removed listener failed")

    def mark_draining(self, worker_id: str) -> None:
        self.pool.set_status(worker_id, WorkerStatus.DRAINING)


class InProcessRegistry(_RegistryBase):
    """Registry for workers in this process: register / deregister directly."""

    def register(self, payload: dict) -> bool:
        return self._upsert(worker_info_from_json(payload))

    def deregister(self, worker_id: str) -> None:
        self._remove(worker_id)

    async def start(self) -> None:  # symmetry with EtcdRegistry
        return None

    async def stop(self) -> None:
        return None


class EtcdRegistry(_RegistryBase):
    def __init__(self, endpoint: str, prefix: str = DEFAULT_PREFIX, pool: WorkerPool | None = None,
                 reconnect_s: float = 1.0) -> None:
        super().__init__(pool)
        self.base = normalize_endpoint(endpoint)
        self.prefix = prefix
        self.reconnect_s = reconnect_s
        self._http = httpx.AsyncClient(base_url=self.base, timeout=httpx.Timeout(10.0, read=None))
        self._task: asyncio.Task | None = None
        self._rev = 0
        self.ready = asyncio.Event()

    async def _snapshot(self) -> None:
        r = await self._http.post("/v3/kv/range", json={"key": b64(self.prefix),
                                                        "range_end": b64(prefix_range_end(self.prefix))})
        r.raise_for_status()
        data = r.json()
        self._rev = int(data.get("header", {}).get("revision", 0))
        seen = set()
        for kv in data.get("kvs", []) or []:
            try:
                w = worker_info_from_json(json.loads(unb64(kv["value"])))
            except Exception:
                logger.warning("skipping malformed worker record %s", kv.get("key"))
                continue
            seen.add(w.worker_id)
            self._upsert(w)
        # records that disappeared while we were not watching
        for w in list(self.pool.all()):
            if w.worker_id not in seen:
                self._remove(w.worker_id)

    def _key_to_id(self, key: bytes) -> str:
        k = key.decode(errors="replace")
        return k[len(self.prefix):] if k.startswith(self.prefix) else k

    def _apply(self, msg: dict) -> None:
        result = msg.get("result", msg)
        for ev in result.get("events") or []:
            kv = ev.get("kv") or {}
            key = unb64(kv.get("key", ""))
            if ev.get("type", "PUT") == "DELETE":
                self._remove(self._key_to_id(key))
            else:
                try:
                    self._upsert(worker_info_from_json(json.loads(unb64(kv.get("value", "")))))
                except Exception:
                    logger.warning("skipping malformed worker record in watch event")
            mr = int(kv.get("mod_revision", 0) or 0)
            self._rev = max(self._rev, mr)

    async def _watch_once(self) -> None:
        body = {"create_request": {"key": b64(self.prefix), "range_end": b64(prefix_range_end(self.prefix)),
                                   "start_revision": str(self._rev + 1)}}
        async with self._http.stream("POST", "/v3/watch", json=body) as resp:
            resp.raise_for_status()
            async for line in resp.aiter_lines():
                line = line.strip()
                if line:
                    self._apply(json.loads(line))

    async def _run(self) -> None:
        while True:
            try:
                await self._snapshot()
                self.ready.set()
                await self._watch_once()
            except asyncio.CancelledError:
                raise
            except Exception as e:  # broken stream / etcd down: back off, resnapshot
                logger.warning("etcd watch failed (%s); retrying", e)
            await asyncio.sleep(self.reconnect_s)

    async def start(self) -> None:
        self._task = asyncio.create_task(self._run())
        try:
            await asyncio.wait_for(self.ready.wait(), timeout=10.0)
        except asyncio.TimeoutError:
            logger.warning("etcd registry not ready after 10 s; continuing")

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except (asyncio.CancelledError, Exception):
                pass
        await self._http.aclose()

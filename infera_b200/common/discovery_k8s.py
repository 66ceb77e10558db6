"""Kubernetes discovery: Pods are the registry.

Pods matching a label selector that carry the annotation
``infera.amd.com/worker-info`` (the JSON registration record) are workers.
A Pod with a ``deletionTimestamp`` is marked DRAINING: kept in the pool (its
in-flight streams finish) but no longer routed. A DELETED event, or the
annotation disappearing, removes the worker. The watch resumes from the
last resource version; when it breaks, a full re-list reconciles deletes
the watch missed. Behaviour of ``infera/common/discovery_k8s.py:43-382``.
"""

from __future__ import annotations

import asyncio
import json
import logging

from infera_b200.common.discovery import _RegistryBase
from infera_b200.common.worker_pool import WorkerStatus, worker_info_from_json

logger = logging.getLogger(__name__)

WORKER_INFO_ANNOTATION = "infera.amd.com/worker-info"


class KubernetesRegistry(_RegistryBase):
    def __init__(self, api, label_selector: str, namespace: str | None = None, pool=None,
                 reconnect_s: float = 1.0) -> None:
        super().__init__(pool)
        from infera_b200.common.k8s_client import in_cluster_namespace

        self.api = api
        self.selector = label_selector
        self.namespace = namespace or in_cluster_namespace()
        self.reconnect_s = reconnect_s
        self._pod_worker: dict[str, str] = {}
        self._rv = "0"
        self._task: asyncio.Task | None = None
        self.ready = asyncio.Event()
        self.relists = 0

    # ------------------------------------------------------------------ pods
    @staticmethod
    def _record(pod: dict) -> dict | None:
        raw = ((pod.get("metadata") or {}).get("annotations") or {}).get(WORKER_INFO_ANNOTATION)
        if not raw:
            return None
        try:
            return json.loads(raw)
        except ValueError:
            logger.warning("pod %s has a malformed worker record", pod["metadata"].get("name"))
            return None

    def _handle(self, kind: str, pod: dict) -> None:
        name = pod["metadata"]["name"]
        rec = self._record(pod)
        if kind == "DELETED" or rec is None:
            wid = self._pod_worker.pop(name, None)
            if wid is not None:
                self._remove(wid)
            return
        try:
            w = worker_info_from_json(rec)
        except Exception:
            logger.warning("pod %s: bad worker record", name)
            return
        old = self._pod_worker.get(name)
        if old is not None and old != w.worker_id:
            self._remove(old)
        if pod["metadata"].get("deletionTimestamp"):
            # terminating: keep (in-flight finishes) but stop routing
            if self.pool.get(w.worker_id) is None:
                if not self._upsert(w):
                    return
            self._pod_worker[name] = w.worker_id
            self.mark_draining(w.worker_id)
            return
        if self._upsert(w):
            self._pod_worker[name] = w.worker_id
            if self.pool.get(w.worker_id).status != WorkerStatus.ACTIVE:
                self.pool.set_status(w.worker_id, WorkerStatus.ACTIVE)

    async def relist(self) -> None:
        data = await self.api.list_pods(self.namespace, self.selector)
        self._rv = str((data.get("metadata") or {}).get("resourceVersion", "0"))
        seen = set()
        for pod in data.get("items") or []:
            seen.add(pod["metadata"]["name"])
            self._handle("ADDED", pod)
        for name in [n for n in self._pod_worker if n not in seen]:
            self._remove(self._pod_worker.pop(name))
        self.relists += 1

    async def _run(self) -> None:
        while True:
            try:
                await self.relist()
                self.ready.set()
                async for ev in self.api.watch_pods(self.namespace, self.selector, self._rv):
                    obj = ev.get("object") or {}
                    if ev.get("type") == "BOOKMARK":
                        self._rv = str(obj.get("metadata", {}).get("resourceVersion", self._rv))
                        continue
                    if ev.get("type") == "ERROR":
                        break
                    self._rv = str(obj.get("metadata", {}).get("resourceVersion", self._rv))
                    self._handle(ev.get("type", "MODIFIED"), obj)
            except asyncio.CancelledError:
                raise
            except Exception as e:
                logger.warning("kubernetes watch failed (%s); re-listing", e)
            await asyncio.sleep(self.reconnect_s)

    async def start(self) -> None:
        self._task = asyncio.create_task(self._run())
        try:
            await asyncio.wait_for(self.ready.wait(), timeout=10.0)
        except asyncio.TimeoutError:
            logger.warning("kubernetes registry not ready after 10 s; continuing")

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except (asyncio.CancelledError, Exception):
                pass

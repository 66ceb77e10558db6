"""Worker-side registration on Kubernetes: the worker writes its record into
its own Pod's ``infera.amd.com/worker-info`` annotation (merge patch),
re-writes it every ``refresh_s`` (30 s: survives an annotation wiped by a
controller), and removes it on deregister before draining. Pod name and
namespace come from the downward API (``POD_NAME`` / ``POD_NAMESPACE``).
Lifecycle of ``infera/common/registration_k8s.py:38-138``.
"""

from __future__ import annotations

import asyncio
import json
import logging
import os

from infera_b200.common.discovery_k8s import WORKER_INFO_ANNOTATION

logger = logging.getLogger(__name__)


class K8sRegistration:
    def __init__(self, api, payload: dict, pod_name: str | None = None, namespace: str | None = None,
                 refresh_s: float = 30.0):
        self.api = api
        self.payload = payload
        self.pod = pod_name or os.environ.get("POD_NAME") or os.environ.get("HOSTNAME", "")
        self.namespace = namespace or os.environ.get("POD_NAMESPACE", "default")
        self.refresh_s = refresh_s
        self.writes = 0

    async def register(self) -> None:
        await self.api.patch_pod(self.namespace, self.pod,
                                 {"metadata": {"annotations": {WORKER_INFO_ANNOTATION: json.dumps(self.payload)}}})
        self.writes += 1

    async def heartbeat_loop(self) -> None:
        while True:
            await asyncio.sleep(self.refresh_s)
            try:
                await self.register()
            except Exception as e:
                logger.warning("refreshing the worker annotation failed: %s", e)

    async def deregister(self) -> None:
        try:
            await self.api.patch_pod(self.namespace, self.pod,
                                     {"metadata": {"annotations": {WORKER_INFO_ANNOTATION: None}}})
        except Exception as e:
            logger.warning("removing the worker annotation failed: %s", e)

    async def close(self) -> None:
        return None

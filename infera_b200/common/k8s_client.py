"""Minimal Kubernetes API access for discovery, registration and scaling.

:class:`InClusterClient` talks to the API server with the Pod's service
account (token, CA and namespace under
``/var/run/secrets/kubernetes.io/serviceaccount``; host from
``KUBERNETES_SERVICE_HOST`` / ``_PORT``). :class:`FakeK8sClient` keeps Pods
and custom resources in memory with resource versions and a watch stream;
tests and the CPU fleet use it (no cluster is reachable here). Both expose:

    list_pods(namespace, label_selector) -> {"metadata": {"resourceVersion"}, "items": [pod]}
    watch_pods(namespace, label_selector, resource_version) -> async iterator of
        {"type": "ADDED"|"MODIFIED"|"DELETED", "object": pod}
    patch_pod(namespace, name, merge_patch)
    get_cr(group, version, namespace, plural, name) / patch_cr(..., merge_patch)

Role of ``infera/common/k8s_client.py:52``.
"""

from __future__ import annotations

import asyncio
import copy
import json
import os
from typing import AsyncIterator

SA_DIR = "/var/run/secrets/kubernetes.io/serviceaccount"


def in_cluster_namespace(default: str = "default") -> str:
    try:
        with open(os.path.join(SA_DIR, "namespace")) as f:
            return f.read().strip() or default
    except OSError:
        return os.environ.get("POD_NAMESPACE", default)


def _selector_matches(labels: dict, selector: str) -> bool:
    for term in (t.strip() for t in selector.split(",") if t.strip()):
        if "!=" in term:
            k, v = term.split("!=", 1)
            if labels.get(k.strip()) == v.strip():
                return False
        elif "=" in term:
            k, v = term.replace("==", "=").split("=", 1)
            if labels.get(k.strip()) != v.strip():
                return False
        elif labels.get(term) is None:
            return False
    return True


def merge_patch(target: dict, patch: dict) -> dict:
    """RFC 7386 JSON merge patch (None deletes a key)."""
    for k, v in patch.items():
        if v is None:
            target.pop(k, None)
        elif isinstance(v, dict) and isinstance(target.get(k), dict):
            merge_patch(target[k], v)
        else:
            target[k] = copy.deepcopy(v)
    return target


class InClusterClient:
    def __init__(self, base_url: str | None = None, token: str | None = None, ca: str | None = None):
        import httpx

        host = os.environ.get("KUBERNETES_SERVICE_HOST", "kubernetes.default.svc")
        port = os.environ.get("KUBERNETES_SERVICE_PORT", "443")
        self.base = base_url or f"https://{host}:{port}"
        if token is None:
            try:
                with open(os.path.join(SA_DIR, "token")) as f:
                    token = f.read().strip()
            except OSError:
                token = None
        ca = ca or os.path.join(SA_DIR, "ca.crt")
        verify = ca if os.path.exists(ca) else True
        headers = {"Authorization": f"Bearer {token}"} if token else {}
        self._http = httpx.AsyncClient(base_url=self.base, headers=headers, verify=verify,
                                       timeout=httpx.Timeout(30.0, read=None))

    async def list_pods(self, namespace: str, label_selector: str) -> dict:
        r = await self._http.get(f"/api/v1/namespaces/{namespace}/pods", params={"labelSelector": label_selector})
        r.raise_for_status()
        return r.json()

    async def watch_pods(self, namespace: str, label_selector: str, resource_version: str
                         ) -> AsyncIterator[dict]:
        params = {"labelSelector": label_selector, "watch": "true", "resourceVersion": resource_version,
                  "allowWatchBookmarks": "true"}
        async with self._http.stream("GET", f"/api/v1/namespaces/{namespace}/pods", params=params) as r:
            r.raise_for_status()
            async for line in r.aiter_lines():
                if line.strip():
                    yield json.loads(line)

    async def patch_pod(self, namespace: str, name: str, patch: dict) -> dict:
        r = await self._http.patch(f"/api/v1/namespaces/{namespace}/pods/{name}", content=json.dumps(patch),
                                   headers={"Content-Type": "application/merge-patch+json"})
        r.raise_for_status()
        return r.json()

    async def get_cr(self, group: str, version: str, namespace: str, plural: str, name: str) -> dict:
        r = await self._http.get(f"/apis/{group}/{version}/namespaces/{namespace}/{plural}/{name}")
        r.raise_for_status()
        return r.json()

    async def patch_cr(self, group: str, version: str, namespace: str, plural: str, name: str, patch: dict) -> dict:
        r = await self._http.patch(f"/apis/{group}/{version}/namespaces/{namespace}/{plural}/{name}",
                                   content=json.dumps(patch), headers={"Content-Type": "application/merge-patch+json"})
        r.raise_for_status()
        return r.json()

    async def aclose(self) -> None:
        await self._http.aclose()


class FakeK8sClient:
    """In-memory API server: Pods, custom resources, resource versions, watches."""

    def __init__(self) -> None:
        self.rv = 1
        self.pods: dict[tuple[str, str], dict] = {}
        self.crs: dict[tuple, dict] = {}
        self._watchers: list[tuple[str, str, asyncio.Queue]] = []
        self.patches = 0
        self.log: list[tuple[int, str, dict]] = []     # (resource version, type, pod) for watch resumes

    def _bump(self, obj: dict) -> None:
        self.rv += 1
        obj.setdefault("metadata", {})["resourceVersion"] = str(self.rv)

    def _emit(self, kind: str, pod: dict) -> None:
        ns = pod["metadata"].get("namespace", "default")
        self.log.append((int(pod["metadata"]["resourceVersion"]), kind, copy.deepcopy(pod)))
        for wns, sel, q in list(self._watchers):
            if wns == ns and _selector_matches(pod["metadata"].get("labels") or {}, sel):
                q.put_nowait({"type": kind, "object": copy.deepcopy(pod)})

    # test helpers ------------------------------------------------------
    def create_pod(self, namespace: str, name: str, labels: dict, annotations: dict | None = None,
                   ip: str = "127.0.0.1") -> dict:
        pod = {"metadata": {"name": name, "namespace": namespace, "labels": dict(labels),
                            "annotations": dict(annotations or {})}, "status": {"podIP": ip, "phase": "Running"}}
        self._bump(pod)
        self.pods[(namespace, name)] = pod
        self._emit("ADDED", pod)
        return pod

    def mark_terminating(self, namespace: str, name: str) -> None:
        pod = self.pods[(namespace, name)]
        pod["metadata"]["deletionTimestamp"] = "2026-01-01T00:00:00Z"
        self._bump(pod)
        self._emit("MODIFIED", pod)

    def delete_pod(self, namespace: str, name: str, silent: bool = False) -> None:
        pod = self.pods.pop((namespace, name))
        self._bump(pod)
        if not silent:  # silent: the watch misses the delete (a re-list must catch it)
            self._emit("DELETED", pod)

    def events_since(self, namespace: str, label_selector: str, resource_version: str) -> list[dict]:
        """Logged events after ``resource_version`` (a watch resuming there
        replays them before following new ones)."""
        try:
            rv = int(resource_version or 0)
        except ValueError:
            rv = 0
        return [{"type": k, "object": copy.deepcopy(p)} for r, k, p in self.log
                if r > rv and p["metadata"].get("namespace", "default") == namespace
                and _selector_matches(p["metadata"].get("labels") or {}, label_selector)]

    def break_watches(self) -> None:
        for _, _, q in self._watchers:
            q.put_nowait(None)

    # API ----------------------------------------------------------------
    async def list_pods(self, namespace: str, label_selector: str) -> dict:
        items = [copy.deepcopy(p) for (ns, _), p in self.pods.items()
                 if ns == namespace and _selector_matches(p["metadata"].get("labels") or {}, label_selector)]
        return {"metadata": {"resourceVersion": str(self.rv)}, "items": items}

    async def watch_pods(self, namespace: str, label_selector: str, resource_version: str):
        q: asyncio.Queue = asyncio.Queue()
        entry = (namespace, label_selector, q)
        self._watchers.append(entry)
        try:
            while True:
                ev = await q.get()
                if ev is None:
                    return
                yield ev
        finally:
            self._watchers.remove(entry)

    async def patch_pod(self, namespace: str, name: str, patch: dict) -> dict:
        pod = self.pods[(namespace, name)]
        merge_patch(pod, patch)
        self._bump(pod)
        self.patches += 1
        self._emit("MODIFIED", pod)
        return copy.deepcopy(pod)

    async def get_cr(self, group, version, namespace, plural, name) -> dict:
        key = (group, version, namespace, plural, name)
        if key not in self.crs:
            raise KeyError(f"{plural}/{name} not found")
        return copy.deepcopy(self.crs[key])

    async def patch_cr(self, group, version, namespace, plural, name, patch) -> dict:
        cr = self.crs[(group, version, namespace, plural, name)]
        merge_patch(cr, patch)
        self._bump(cr)
        return copy.deepcopy(cr)

    async def aclose(self) -> None:
        return None

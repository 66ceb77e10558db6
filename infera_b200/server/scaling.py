"""``GET|POST /v1/admin/scale``: read and patch the replica counts of an
``InferaDeployment`` custom resource (``spec.services.<name>.replicas``).

One merge-patch per request changes every named service atomically; a
service name that does not exist is a 404, a non-integer or negative count
a 400, and scaling every worker service of the deployment to 0 is refused
(a deployment that serves nothing is a misconfiguration, not a scale-down;
``infera/server/scaling.py:78-285``). The Kubernetes API is reached through
an injected client (``get_cr`` / ``patch_cr``), which tests fake."""

from __future__ import annotations

GROUP = "infera.amd.com"
VERSION = "v1alpha1"
PLURAL = "inferadeployments"


class ScaleError(Exception):
    def __init__(self, msg: str, status: int = 400):
        super().__init__(msg)
        self.status = status


class DeploymentScaler:
    def __init__(self, api, name: str, namespace: str = "default"):
        self.api = api
        self.name = name
        self.namespace = namespace

    async def _cr(self) -> dict:
        return await self.api.get_cr(GROUP, VERSION, self.namespace, PLURAL, self.name)

    @staticmethod
    def _services(cr: dict) -> dict:
        return (cr.get("spec") or {}).get("services") or {}

    async def get(self) -> dict:
        cr = await self._cr()
        svcs = self._services(cr)
        return {"deployment": self.name, "namespace": self.namespace,
                "services": {n: {"replicas": int(s.get("replicas", 1)), "role": s.get("role"),
                                 "componentType": s.get("componentType")} for n, s in svcs.items()}}

    def _validate(self, cr: dict, want: dict) -> dict:
        svcs = self._services(cr)
        clean = {}
        for name, n in want.items():
            if name not in svcs:
                raise ScaleError(f"unknown service {name!r}", 404)
            if isinstance(n, dict):
                n = n.get("replicas")
            if not isinstance(n, int) or isinstance(n, bool) or n < 0:
                raise ScaleError(f"replicas for {name!r} must be a non-negative integer")
            clean[name] = n
        workers = [k for k, s in svcs.items() if s.get("componentType", "worker") == "worker"]
        after = {k: clean.get(k, int(svcs[k].get("replicas", 1))) for k in workers}
        if workers and all(v == 0 for v in after.values()):
            raise ScaleError("refusing to scale every worker service to 0")
        return clean

    async def scale(self, body: dict) -> dict:
        want = body.get("services") if isinstance(body, dict) else None
        if not isinstance(want, dict) or not want:
            raise ScaleError("body must be {\"services\": {name: replicas}}")
        cr = await self._cr()
        clean = self._validate(cr, want)
        patch = {"spec": {"services": {k: {"replicas": v} for k, v in clean.items()}}}
        await self.api.patch_cr(GROUP, VERSION, self.namespace, PLURAL, self.name, patch)
        return {"deployment": self.name, "scaled": clean}

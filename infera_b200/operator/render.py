"""InferaDeployment custom resource -> Kubernetes manifests, offline.

The same contract as the reference's Go operator
(``deploy/operator/api/v1alpha1/inferadeployment_types.go:52-289``,
``internal/controller/builders.go:576-716``, ``gaie.go:43-396``), as a
pure function from a CR (dict) to manifests (dicts), so it runs and is
tested without a cluster:

* ``spec.services.<name>``: ``componentType`` frontend (the router:
  Deployment + ClusterIP Service) or worker (this framework's engine
  worker: Deployment, or a LeaderWorkerSet when ``numberOfNodes > 1``),
  ``role`` mixed / prefill / decode, ``replicas``, ``resources.gpu`` ->
  ``nvidia.com/gpu``, ``sharedMemory`` -> a memory-backed /dev/shm,
  ``args`` / ``env`` / ``podLabels`` / ``extraPodSpec`` merged in;
* workers get a readiness probe on ``/health`` (unless
  ``skipReadinessProbe``), a preStop sleep of 15 s (the router drops the
  Pod first) and ``terminationGracePeriodSeconds = max(120, 15 + drain
  timeout + 50)`` with the drain timeout from ``INFERA_DRAIN_TIMEOUT``
  (default 30);
* ``discoveryBackend: kubernetes`` adds the ServiceAccount / Role /
  RoleBinding the registry and the self-registration need, and workers
  register through their Pod annotation; ``etcd`` passes the endpoint;
* ``gaie.enabled`` adds the endpoint-picker Deployment + Service, an
  InferencePool over the worker Pods and an HTTPRoute on the gateway;
* ``nats.deploy`` adds a NATS StatefulSet + Service.

``rollup(cr, observed)`` computes the status block from observed replica
counts. ``python -m infera_b200.operator render cr.yaml`` prints the
manifests as multi-document YAML.
"""

from __future__ import annotations

import copy

GROUP = "infera.amd.com"
PRESTOP_S = 15
TEARDOWN_S = 50
GRACE_FLOOR_S = 120
DEFAULT_DRAIN_S = 30
WORKER_PORT = 9000
FRONTEND_PORT = 8000
EPP_PORT = 9002


def _labels(cr: dict, svc: str, extra: dict | None = None) -> dict:
    name = cr["metadata"]["name"]
    lab = {"app.kubernetes.io/name": "infera-b200", "app.kubernetes.io/instance": name,
           f"{GROUP}/deployment": name, f"{GROUP}/service": svc}
    lab.update(extra or {})
    return lab


def _env(items: list | None) -> list:
    return [copy.deepcopy(e) for e in (items or [])]


def drain_timeout(spec_env: list, svc_env: list) -> int:
    v = DEFAULT_DRAIN_S
    for e in list(spec_env or []) + list(svc_env or []):  # service overrides deployment
        if e.get("name") == "INFERA_DRAIN_TIMEOUT":
            try:
                v = int(float(e.get("value", v)))
            except (TypeError, ValueError):
                pass
    return v


def grace_seconds(drain_s: int) -> int:
    return max(GRACE_FLOOR_S, PRESTOP_S + drain_s + TEARDOWN_S)


def _merge_pod_spec(base: dict, extra: dict | None) -> dict:
    if not extra:
        return base
    out = copy.deepcopy(base)
    for k, v in extra.items():
        if k == "containers":
            # extra containers are sidecars; a container named like ours patches it
            names = {c["name"]: c for c in out["containers"]}
            for c in v:
                if c.get("name") in names:
                    names[c["name"]].update(copy.deepcopy(c))
                else:
                    out["containers"].append(copy.deepcopy(c))
        elif k == "volumes":
            out.setdefault("volumes", []).extend(copy.deepcopy(v))
        else:
            out[k] = copy.deepcopy(v)
    return out


def _discovery_args(spec: dict) -> list[str]:
    if spec.get("discoveryBackend", "etcd") == "kubernetes":
        return []
    ep = spec.get("etcdEndpoint")
    if not ep:
        raise ValueError("discoveryBackend etcd needs spec.etcdEndpoint")
    return ["--etcd-endpoint", ep]


def _worker(cr: dict, name: str, s: dict) -> list[dict]:
    spec = cr["spec"]
    ns = cr["metadata"].get("namespace", "default")
    full = f"{cr['metadata']['name']}-{name}"
    role = s.get("role", "mixed")
    port = int(s.get("port") or WORKER_PORT)
    res = s.get("resources") or {}
    gpus = int(res.get("gpu", 1))
    labels = _labels(cr, name, {f"{GROUP}/role": role, f"{GROUP}/component": "worker", **(s.get("podLabels") or {})})
    args = ["python", "-m", "infera_b200.engine.worker", "--host", "0.0.0.0", "--port", str(port),
            "--disagg-mode", role, "--advertise-host", "$(POD_IP)"]
    if spec.get("discoveryBackend", "etcd") == "kubernetes":
        args.append("--k8s-register")
    else:
        args += _discovery_args(spec)
    args += list(s.get("args") or [])
    drain = drain_timeout(spec.get("envs"), s.get("env"))
    args += ["--drain-timeout", str(drain)]
    limits = {"nvidia.com/gpu": str(gpus)}
    if res.get("cpu"):
        limits["cpu"] = str(res["cpu"])
    if res.get("memory"):
        limits["memory"] = str(res["memory"])
    env = [{"name": "POD_NAME", "valueFrom": {"fieldRef": {"fieldPath": "metadata.name"}}},
           {"name": "POD_NAMESPACE", "valueFrom": {"fieldRef": {"fieldPath": "metadata.namespace"}}},
           {"name": "POD_IP", "valueFrom": {"fieldRef": {"fieldPath": "status.podIP"}}}]
    env += _env(spec.get("envs")) + _env(s.get("env"))
    container = {"name": "worker", "image": s.get("image") or spec.get("image", "infera-b200:latest"),
                 "command": args, "ports": [{"name": "http", "containerPort": port}], "env": env,
                 "resources": {"limits": limits, "requests": dict(limits)},
                 "lifecycle": {"preStop": {"exec": {"command": ["sleep", str(PRESTOP_S)]}}}}
    if not s.get("skipReadinessProbe"):
        container["readinessProbe"] = {"httpGet": {"path": "/health", "port": port}, "periodSeconds": 5,
                                       "failureThreshold": 3}
    pod = {"containers": [container], "terminationGracePeriodSeconds": grace_seconds(drain)}
    if spec.get("discoveryBackend", "etcd") == "kubernetes":
        pod["serviceAccountName"] = f"{cr['metadata']['name']}-infera"
    shm = res.get("sharedMemory") or s.get("sharedMemory")
    if shm:
        pod["volumes"] = [{"name": "shm", "emptyDir": {"medium": "Memory", "sizeLimit": shm}}]
        container["volumeMounts"] = [{"name": "shm", "mountPath": "/dev/shm"}]
    pod = _merge_pod_spec(pod, s.get("extraPodSpec"))
    replicas = int(s.get("replicas", 1))
    template = {"metadata": {"labels": labels}, "spec": pod}
    nodes = int(s.get("numberOfNodes") or 1)
    if nodes > 1:
        return [{"apiVersion": "leaderworkerset.x-k8s.io/v1", "kind": "LeaderWorkerSet",
                 "metadata": {"name": full, "namespace": ns, "labels": labels},
                 "spec": {"replicas": replicas, "leaderWorkerTemplate": {"size": nodes, "workerTemplate": template}}}]
    return [{"apiVersion": "apps/v1", "kind": "Deployment", "metadata": {"name": full, "namespace": ns, "labels": labels},
             "spec": {"replicas": replicas, "selector": {"matchLabels": {f"{GROUP}/deployment": cr["metadata"]["name"],
                                                                         f"{GROUP}/service": name}},
                      "strategy": {"type": "RollingUpdate", "rollingUpdate": {"maxUnavailable": 0, "maxSurge": 1}},
                      "template": template}}]


def _frontend(cr: dict, name: str, s: dict) -> list[dict]:
    spec = cr["spec"]
    ns = cr["metadata"].get("namespace", "default")
    full = f"{cr['metadata']['name']}-{name}"
    port = int(s.get("port") or FRONTEND_PORT)
    labels = _labels(cr, name, {f"{GROUP}/component": "frontend", **(s.get("podLabels") or {})})
    disc = spec.get("discoveryBackend", "etcd")
    args = ["python", "-m", "infera_b200.server", "--host", "0.0.0.0", "--port", str(port),
            "--discovery-backend", disc]
    if disc == "kubernetes":
        args += ["--k8s-label-selector", f"{GROUP}/deployment={cr['metadata']['name']},{GROUP}/component=worker"]
    else:
        args += _discovery_args(spec)
    args += list(s.get("args") or [])
    container = {"name": "router", "image": s.get("image") or spec.get("image", "infera-b200:latest"),
                 "command": args, "ports": [{"name": "http", "containerPort": port}],
                 "env": _env(spec.get("envs")) + _env(s.get("env")),
                 "readinessProbe": {"httpGet": {"path": "/health", "port": port}, "periodSeconds": 5}}
    pod = {"containers": [container]}
    if disc == "kubernetes":
        pod["serviceAccountName"] = f"{cr['metadata']['name']}-infera"
    pod = _merge_pod_spec(pod, s.get("extraPodSpec"))
    sel = {f"{GROUP}/deployment": cr["metadata"]["name"], f"{GROUP}/service": name}
    return [{"apiVersion": "apps/v1", "kind": "Deployment", "metadata": {"name": full, "namespace": ns, "labels": labels},
             "spec": {"replicas": int(s.get("replicas", 1)), "selector": {"matchLabels": sel},
                      "template": {"metadata": {"labels": labels}, "spec": pod}}},
            {"apiVersion": "v1", "kind": "Service", "metadata": {"name": full, "namespace": ns, "labels": labels},
             "spec": {"selector": sel, "ports": [{"name": "http", "port": port, "targetPort": port}]}}]


def _rbac(cr: dict) -> list[dict]:
    ns = cr["metadata"].get("namespace", "default")
    sa = f"{cr['metadata']['name']}-infera"
    return [{"apiVersion": "v1", "kind": "ServiceAccount", "metadata": {"name": sa, "namespace": ns}},
            {"apiVersion": "rbac.authorization.k8s.io/v1", "kind": "Role", "metadata": {"name": sa, "namespace": ns},
             "rules": [{"apiGroups": [""], "resources": ["pods"], "verbs": ["get", "list", "watch", "patch"]},
                       {"apiGroups": [GROUP], "resources": ["inferadeployments"], "verbs": ["get", "patch"]}]},
            {"apiVersion": "rbac.authorization.k8s.io/v1", "kind": "RoleBinding",
             "metadata": {"name": sa, "namespace": ns},
             "roleRef": {"apiGroup": "rbac.authorization.k8s.io", "kind": "Role", "name": sa},
             "subjects": [{"kind": "ServiceAccount", "name": sa, "namespace": ns}]}]


def _gaie(cr: dict) -> list[dict]:
    g = cr["spec"]["gaie"]
    ns = cr["metadata"].get("namespace", "default")
    name = cr["metadata"]["name"]
    epp = f"{name}-epp"
    pool = f"{name}-pool"
    disc = cr["spec"].get("discoveryBackend", "etcd")
    args = ["python", "-m", "infera_b200.gaie", "--port", str(EPP_PORT), "--discovery-backend", disc]
    if disc == "kubernetes":
        args += ["--k8s-label-selector", f"{GROUP}/deployment={name},{GROUP}/component=worker"]
    else:
        args += _discovery_args(cr["spec"])
    fport = int(g.get("frontendPort") or FRONTEND_PORT)
    args += ["--target-port", str(fport)]
    labels = _labels(cr, "epp", {f"{GROUP}/component": "epp"})
    sel = {f"{GROUP}/deployment": name, f"{GROUP}/component": "epp"}
    out = [{"apiVersion": "apps/v1", "kind": "Deployment", "metadata": {"name": epp, "namespace": ns, "labels": labels},
            "spec": {"replicas": 1, "selector": {"matchLabels": sel},
                     "template": {"metadata": {"labels": labels},
                                  "spec": {"containers": [{"name": "epp", "image": g.get("eppImage") or
                                                           cr["spec"].get("image", "infera-b200:latest"),
                                                           "command": args,
                                                           "ports": [{"name": "grpc", "containerPort": EPP_PORT}]}],
                                           **({"serviceAccountName": f"{name}-infera"} if disc == "kubernetes"
                                              else {})}}}},
           {"apiVersion": "v1", "kind": "Service", "metadata": {"name": epp, "namespace": ns, "labels": labels},
            "spec": {"selector": sel, "ports": [{"name": "grpc", "port": EPP_PORT, "targetPort": EPP_PORT,
                                                 "appProtocol": "http2"}]}},
           {"apiVersion": "inference.networking.x-k8s.io/v1alpha2", "kind": "InferencePool",
            "metadata": {"name": pool, "namespace": ns},
            "spec": {"targetPortNumber": fport,
                     "selector": {f"{GROUP}/deployment": name, f"{GROUP}/component": "worker"},
                     "extensionRef": {"name": epp, "portNumber": EPP_PORT, "failureMode": "FailClose"}}}]
    route = {"apiVersion": "gateway.networking.k8s.io/v1", "kind": "HTTPRoute",
             "metadata": {"name": f"{name}-route", "namespace": ns},
             "spec": {"parentRefs": [{"name": g["gatewayName"],
                                      **({"namespace": g["gatewayNamespace"]} if g.get("gatewayNamespace") else {})}],
                      "rules": [{"matches": [{"path": {"type": "PathPrefix", "value": "/v1"}}],
                                 "backendRefs": [{"group": "inference.networking.x-k8s.io", "kind": "InferencePool",
                                                  "name": pool}]}]}}
    if g.get("hostnames"):
        route["spec"]["hostnames"] = list(g["hostnames"])
    out.append(route)
    return out


def _nats(cr: dict) -> list[dict]:
    n = cr["spec"]["nats"]
    ns = cr["metadata"].get("namespace", "default")
    name = f"{cr['metadata']['name']}-nats"
    labels = _labels(cr, "nats")
    sts = {"apiVersion": "apps/v1", "kind": "StatefulSet", "metadata": {"name": name, "namespace": ns, "labels": labels},
           "spec": {"serviceName": name, "replicas": 1, "selector": {"matchLabels": labels},
                    "template": {"metadata": {"labels": labels},
                                 "spec": {"containers": [{"name": "nats", "image": n.get("image", "nats:2.10"),
                                                          "args": ["-js", "-sd", "/data"],
                                                          "ports": [{"name": "client", "containerPort": 4222}],
                                                          "volumeMounts": [{"name": "data", "mountPath": "/data"}]}]}},
                    "volumeClaimTemplates": [{"metadata": {"name": "data"},
                                              "spec": {"accessModes": ["ReadWriteOnce"],
                                                       "resources": {"requests": {"storage": n.get("storageSize",
                                                                                                   "10Gi")}},
                                                       **({"storageClassName": n["storageClassName"]}
                                                          if n.get("storageClassName") else {})}}]}}
    svc = {"apiVersion": "v1", "kind": "Service", "metadata": {"name": name, "namespace": ns, "labels": labels},
           "spec": {"selector": labels, "ports": [{"name": "client", "port": 4222}]}}
    return [sts, svc]


def render(cr: dict) -> list[dict]:
    if cr.get("kind") != "InferaDeployment":
        raise ValueError("not an InferaDeployment")
    spec = cr.get("spec") or {}
    services = spec.get("services") or {}
    if not services:
        raise ValueError("spec.services is empty")
    out: list[dict] = []
    if spec.get("discoveryBackend", "etcd") == "kubernetes":
        out += _rbac(cr)
    for name in sorted(services):
        s = services[name]
        ct = s.get("componentType")
        if ct == "worker":
            out += _worker(cr, name, s)
        elif ct in ("frontend", "server"):
            out += _frontend(cr, name, s)
        else:
            raise ValueError(f"service {name}: unknown componentType {ct!r}")
    if (spec.get("gaie") or {}).get("enabled"):
        out += _gaie(cr)
    if (spec.get("nats") or {}).get("deploy"):
        out += _nats(cr)
    owner = {"apiVersion": f"{GROUP}/v1alpha1", "kind": "InferaDeployment", "name": cr["metadata"]["name"],
             "uid": cr["metadata"].get("uid", ""), "controller": True}
    for m in out:
        m["metadata"].setdefault("ownerReferences", [owner])
    return out


def rollup(cr: dict, observed: dict[str, tuple[int, int]]) -> dict:
    """``observed``: service -> (replicas, ready replicas)."""
    services = {}
    ready = True
    failed = False
    for name, s in (cr["spec"].get("services") or {}).items():
        want = int(s.get("replicas", 1))
        have, rdy = observed.get(name, (0, 0))
        kind = "LeaderWorkerSet" if int(s.get("numberOfNodes") or 1) > 1 else "Deployment"
        services[name] = {"kind": kind, "replicas": have, "readyReplicas": rdy}
        ready = ready and rdy >= want
        failed = failed or (want > 0 and have == 0 and name in observed)
    state = "Ready" if ready else ("Failed" if failed else "Progressing")
    return {"observedGeneration": cr["metadata"].get("generation", 0), "state": state, "services": services,
            "conditions": [{"type": "Ready", "status": "True" if ready else "False", "reason": state}]}


def to_yaml(manifests: list[dict]) -> str:
    import yaml

    return "---\n".join(yaml.safe_dump(m, sort_keys=False) for m in manifests)

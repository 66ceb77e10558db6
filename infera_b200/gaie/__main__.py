"""``python -m infera_b200.gaie``: the endpoint-picker process for a GAIE
gateway. Discovery (etcd or Kubernetes) and the KV-aware policy as in the
router; serves ext_proc gRPC on ``--port`` (default 9002). Role of
``infera/gaie/__main__.py``."""

from __future__ import annotations

import argparse
import asyncio
import logging


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="python -m infera_b200.gaie")
    ap.add_argument("--port", type=int, default=9002)
    ap.add_argument("--discovery-backend", choices=("etcd", "kubernetes"), default="etcd")
    ap.add_argument("--etcd-endpoint", default=None)
    ap.add_argument("--k8s-label-selector", default=None)
    ap.add_argument("--k8s-namespace", default=None)
    ap.add_argument("--target-port", type=int, default=None, help="InferencePool target port on the worker pods")
    ap.add_argument("--router-policy", default="kv-aware")
    a = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO)

    async def run():
        from infera_b200.gaie.extproc import serve
        from infera_b200.gaie.picker import EndpointPicker
        from infera_b200.router.breaker import CircuitBreaker
        from infera_b200.router.policy.factory import build_policy

        if a.discovery_backend == "etcd":
            from infera_b200.common.discovery import EtcdRegistry

            reg = EtcdRegistry(a.etcd_endpoint)
        else:
            from infera_b200.common.discovery_k8s import KubernetesRegistry
            from infera_b200.common.k8s_client import InClusterClient

            reg = KubernetesRegistry(InClusterClient(), a.k8s_label_selector, a.k8s_namespace)
        policy = build_policy(a.router_policy)
        reg.on_worker_added(policy.on_worker_added)
        reg.on_worker_removed(lambda w: policy.on_worker_removed(w.worker_id))
        await reg.start()
        srv, _, _ = await serve(EndpointPicker(reg.pool, policy, a.target_port, CircuitBreaker()), port=a.port)
        await srv.wait_for_termination()

    asyncio.run(run())


if __name__ == "__main__":
    main()

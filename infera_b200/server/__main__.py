"""``python -m infera_b200.server``: the router process.

Builds the policy (KV-aware: tokenizer + KV-event client), the breaker and
metrics, the tier-aware KV index plane (index, writer, per-worker
subscribers, snapshot reconciler), the registry (etcd gateway, Kubernetes, or in-process) whose
add/remove callbacks feed the policy, then the Auto or Direct router and the
FastAPI app, and serves it with uvicorn. ``--router-backend native`` execs
the C++ router binary instead (same flags where supported). Structure of
``infera/server/__main__.py:39-327``.
"""

from __future__ import annotations

import asyncio
import logging
import os
import sys

from infera_b200.server.args import parse_server_args


def build_router_stack(args, registry=None, transport=None):
    """Everything but the HTTP server; returns the app state. Used by the CLI
    and by in-process fleets / tests."""
    from infera_b200.common.discovery import InProcessRegistry
    from infera_b200.router.auto import AutoRouter
    from infera_b200.router.breaker import CircuitBreaker
    from infera_b200.router.direct import DirectRouter
    from infera_b200.router.policy.factory import build_policy
    from infera_b200.server.app import AppState
    from infera_b200.server.metrics import RouterMetrics
    from infera_b200.server.profiling import ProfileFanout
    from infera_b200.utils.tokenizer import load_tokenizer

    metrics = RouterMetrics()
    tok = load_tokenizer(args.router_tokenizer_path)
    policy = build_policy(args.router_policy, tokenizer=tok, overlap_weight=args.kv_overlap_weight,
                          prefill_overlap_weight=args.kv_prefill_overlap_weight,
                          decode_overlap_weight=args.kv_decode_overlap_weight, metrics=metrics,
                          use_zmq=transport is None and getattr(args, "kv_event_transport", "zmq") == "zmq")
    breaker = CircuitBreaker(args.breaker_failure_threshold, args.breaker_cooldown_s, args.breaker_max_cooldown_s,
                             on_change=metrics.breaker_changed)
    if registry is None:
        if args.discovery_backend == "etcd":
            from infera_b200.common.discovery import EtcdRegistry

            registry = EtcdRegistry(args.etcd_endpoint, args.etcd_prefix)
        elif args.discovery_backend == "kubernetes":
            from infera_b200.common.discovery_k8s import KubernetesRegistry
            from infera_b200.common.k8s_client import InClusterClient

            registry = KubernetesRegistry(InClusterClient(), args.k8s_label_selector, args.k8s_namespace)
        else:
            registry = InProcessRegistry()
    registry.on_worker_added(policy.on_worker_added)
    registry.on_worker_removed(lambda w: (policy.on_worker_removed(w.worker_id), breaker.forget(w.worker_id)))
    # the tier-aware KV index: workers that register a kv block with an
    # events endpoint publish which prefixes they hold in GPU memory, host
    # memory and on disk
    from infera_b200.kv.plane import KvIndexPlane

    kv_plane = KvIndexPlane()
    registry.on_worker_added(kv_plane.on_worker_added)
    registry.on_worker_removed(kv_plane.on_worker_removed)
    kw = dict(breaker=breaker, request_max_retries=args.request_max_retries, migration_limit=args.migration_limit,
              metrics=metrics)
    if transport is None and getattr(args, "request_transport", "http") == "nats":
        from infera_b200.common.nats_wire import NatsBus
        from infera_b200.common.request_transport import BusRequestClient
        from infera_b200.router.transport import RoutingTransport

        # connected by ``serve`` inside the event loop
        transport = RoutingTransport(bus_client=BusRequestClient(NatsBus(args.nats_url),
                                                                 idle_timeout=args.nats_idle_timeout,
                                                                 max_duration=args.nats_max_duration,
                                                                 jetstream=getattr(args, "nats_jetstream", False)))
    if transport is not None:
        kw["transport"] = transport
    router_cls = DirectRouter if args.router_mode == "direct" else AutoRouter
    router = router_cls(registry.pool, policy, **kw)
    profiler = ProfileFanout(registry.pool, router.transport) if args.enable_profiling else None
    scaler = None
    if args.enable_scaling_api and args.scaling_deployment:
        from infera_b200.common.k8s_client import InClusterClient
        from infera_b200.server.scaling import DeploymentScaler

        scaler = DeploymentScaler(InClusterClient(), args.scaling_deployment, args.k8s_namespace or "default")
    kvd = None
    if args.kvd_socket_path:
        from infera_b200.kvd.client import KvdPrefetchClient

        kvd = KvdPrefetchClient(args.kvd_socket_path)
    return AppState(router=router, registry=registry, policy=policy, metrics=metrics, profiler=profiler,
                    scaler=scaler, kvd_client=kvd, block_size=args.block_size, kv_plane=kv_plane)


async def serve(args) -> None:
    import uvicorn

    from infera_b200.server.app import build_app

    state = build_router_stack(args)
    bus = getattr(getattr(state.router.transport, "bus", None), "bus", None)
    if bus is not None:
        await bus.connect()
    kv = getattr(state.policy, "kv_client", None)
    if args.kv_event_transport == "nats" and kv is not None:
        if bus is None:
            from infera_b200.common.nats_wire import NatsBus

            bus = await NatsBus(args.nats_url).connect()
        await kv.attach_nats(bus, jetstream=getattr(args, "nats_jetstream", False))
    await state.kv_plane.start()
    await state.registry.start()
    app = build_app(state)
    cfg = uvicorn.Config(app, host=args.host, port=args.port, log_level=args.log_level, access_log=False)
    server = uvicorn.Server(cfg)
    try:
        await server.serve()
    finally:
        await state.registry.stop()
        await state.kv_plane.stop()
        await state.router.aclose()
        await state.policy.aclose()


def main(argv=None) -> None:
    args = parse_server_args(argv)
    logging.basicConfig(level=getattr(logging, args.log_level.upper(), logging.INFO),
                        format="%(asctime)s %(levelname)s %(name)s: %(message)s")
    for noisy in ("httpx", "httpcore"):
        logging.getLogger(noisy).setLevel(logging.WARNING)
    if args.router_backend == "native":
        from infera_b200.server.launch_native import exec_native

        exec_native(args, sys.argv[1:] if argv is None else argv)
        return
    asyncio.run(serve(args))


if __name__ == "__main__":
    os.environ.setdefault("PYTHONUNBUFFERED", "1")
    main()

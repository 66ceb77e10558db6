"""Router / front-door flags. Precedence: flag > environment > default
(the convention and flag names of ``infera/server/args.py:14-257``)."""

from __future__ import annotations

import argparse
import os

from infera_b200.router.policy.factory import POLICY_NAMES


def _env(name: str, default=None):
    v = os.environ.get(name)
    return default if v in (None, "") else v


def _env_bool(name: str) -> bool:
    return str(os.environ.get(name, "")).lower() in ("1", "true", "yes")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="python -m infera_b200.server", description="infera-b200 router")
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--discovery-backend", choices=("etcd", "kubernetes", "inprocess"),
                   default=_env("INFERA_DISCOVERY_BACKEND", "etcd"))
    p.add_argument("--etcd-endpoint", default=_env("INFERA_ETCD_ENDPOINT"))
    p.add_argument("--etcd-prefix", default="/infera/workers/")
    p.add_argument("--k8s-label-selector", default=_env("INFERA_K8S_LABEL_SELECTOR"))
    p.add_argument("--k8s-namespace", default=None)
    p.add_argument("--request-transport", choices=("http", "nats"), default=_env("INFERA_REQUEST_TRANSPORT", "http"),
                   help="nats: workers registered with request_transport=bus are reached over NATS, others over HTTP")
    p.add_argument("--nats-url", default=_env("INFERA_NATS_URL", "nats://127.0.0.1:4222"))
    p.add_argument("--nats-idle-timeout", type=float, default=900.0)
    p.add_argument("--nats-max-duration", type=float, default=None)
    p.add_argument("--router-backend", choices=("python", "native"), default=_env("INFERA_ROUTER_BACKEND", "python"))
    p.add_argument("--router-mode", choices=("auto", "direct"), default=_env("INFERA_ROUTER_MODE", "auto"))
    p.add_argument("--router-policy", choices=POLICY_NAMES, default="kv-aware")
    p.add_argument("--kv-event-transport", choices=("zmq", "nats"), default=_env("INFERA_KV_EVENT_TRANSPORT", "zmq"),
                   help="nats: KV-event batches arrive on infera.kv.events.> (workers run the NATS relay)")
    p.add_argument("--nats-jetstream", action="store_true", default=_env("INFERA_NATS_JETSTREAM", "") == "1",
                   help="with NATS: KV events from the INFERA_KV_EVENTS stream with views bootstrapped from the "
                        "INFERA_KV_VIEWS bucket; bus requests through the INFERA_REQUESTS work queue")
    p.add_argument("--router-tokenizer-path", default=_env("INFERA_ROUTER_TOKENIZER_PATH"))
    p.add_argument("--kv-overlap-weight", type=float, default=1.0)
    p.add_argument("--kv-prefill-overlap-weight", type=float, default=None)
    p.add_argument("--kv-decode-overlap-weight", type=float, default=None)
    p.add_argument("--kvd-socket-path", default=_env("INFERA_KVD_SOCKET_PATH"))
    p.add_argument("--enable-profiling", action="store_true", default=_env_bool("INFERA_ENABLE_PROFILING"))
    p.add_argument("--enable-scaling-api", action="store_true", default=_env_bool("INFERA_ENABLE_SCALING_API"))
    p.add_argument("--scaling-deployment", default=_env("INFERA_SCALING_DEPLOYMENT"))
    p.add_argument("--request-max-retries", type=int, default=int(_env("INFERA_REQUEST_MAX_RETRIES", "1")))
    p.add_argument("--migration-limit", type=int, default=int(_env("INFERA_MIGRATION_LIMIT", "0")))
    p.add_argument("--breaker-failure-threshold", type=int,
                   default=int(_env("INFERA_BREAKER_FAILURE_THRESHOLD", "3")))
    p.add_argument("--breaker-cooldown-s", type=float, default=float(_env("INFERA_BREAKER_COOLDOWN_S", "5")))
    p.add_argument("--breaker-max-cooldown-s", type=float,
                   default=float(_env("INFERA_BREAKER_MAX_COOLDOWN_S", "60")))
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--log-level", default=_env("INFERA_LOG_LEVEL", "info"))
    return p


def parse_server_args(argv=None) -> argparse.Namespace:
    a = build_parser().parse_args(argv)
    if a.discovery_backend == "etcd" and not a.etcd_endpoint:
        raise SystemExit("--discovery-backend=etcd requires --etcd-endpoint")
    if a.discovery_backend == "kubernetes" and not a.k8s_label_selector:
        raise SystemExit("--discovery-backend=kubernetes requires --k8s-label-selector")
    return a

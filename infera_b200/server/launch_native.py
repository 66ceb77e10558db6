"""``--router-backend native``: replace this process with the C++ router.

The native binary (``infera_b200/lib/ib200_router``, built from
``infera_b200/native/router``) takes the same flags as the Python router
for the features it implements (etcd, Kubernetes or static discovery,
byte, word-level and byte-level BPE tokenizers, KV-aware and
round-robin policies, auto / direct modes, failover, breaker, PD pairs);
Python-only flags are accepted and ignored. Role of the reference's Rust
launcher (``infera/server/__main__.py:323-327`` execs ``rust/router``).
"""

from __future__ import annotations

import os
import sys

from infera_b200.build import ROUTER_BIN, build_router

PY_ONLY = {"--enable-profiling", "--enable-scaling-api"}
PY_ONLY_WITH_VALUE = {"--scaling-deployment", "--kvd-socket-path"}


def native_argv(argv: list[str]) -> list[str]:
    out, skip = [], False
    for a in argv:
        if skip:
            skip = False
            continue
        name = a.split("=", 1)[0]
        if name in PY_ONLY:
            continue
        if name in PY_ONLY_WITH_VALUE:
            skip = "=" not in a
            continue
        out.append(a)
    return out


def router_binary() -> str:
    path = build_router() or ROUTER_BIN
    if not os.path.exists(path):
        raise SystemExit("native router not built (python -m infera_b200.build)")
    return str(path)


def exec_native(args, argv: list[str]) -> None:
    if args.discovery_backend not in ("etcd", "kubernetes"):
        raise SystemExit(f"--router-backend native supports etcd and kubernetes discovery; "
                         f"got {args.discovery_backend!r}")
    binary = router_binary()
    sys.stdout.flush()
    sys.stderr.flush()
    os.execv(binary, [binary, *native_argv(argv)])

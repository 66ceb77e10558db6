"""Launch-time checks for prefill/decode (PD) workers.

This framework moves KV from prefill to decode GPUs with its own NVLink
page push (``b200-nvlink-push``): both instances must be on one NVLink
domain and every prefill GPU must reach every decode GPU peer-to-peer. The
checks fail fast with an actionable message instead of a hang:

* the advertised host must be routable when peers or the router live on
  other machines (wildcard / loopback hosts are fine only on one node);
* the KV endpoint (where the decode pool exports its page-pool handles)
  must be a local ``ipc://`` / filesystem path: there is no cross-node path;
* every (prefill GPU, decode GPU) pair must allow peer access.

Role of ``infera/common/disagg_preflight.py:42-111`` (which checks for RDMA
transports instead).
"""

from __future__ import annotations

from typing import Callable, Iterable

NON_ROUTABLE = frozenset({"", "0.0.0.0", "127.0.0.1", "localhost", "::", "::1"})


class DisaggPreflightError(RuntimeError):
    pass


def is_routable_host(host: str | None) -> bool:
    return host is not None and host.strip().lower() not in NON_ROUTABLE


def validate_advertise_host(host: str | None, *, is_disagg: bool, single_node: bool) -> None:
    if not is_disagg or single_node:
        return
    if not is_routable_host(host):
        raise DisaggPreflightError(
            f"PD worker advertises {host!r}, which peers on other machines cannot reach; pass --advertise-host "
            f"with this machine's address (or run prefill, decode and router on one node)")


def validate_kv_endpoint(endpoint: str | None, *, mode: str) -> None:
    if mode != "decode":
        return
    if not endpoint:
        raise DisaggPreflightError("a decode worker needs --kv-push-endpoint (ipc://... or a socket path) so "
                                   "prefill workers can map its KV page pool")
    if endpoint.startswith(("tcp://", "http://", "https://", "rdma://")):
        raise DisaggPreflightError(f"KV push endpoint {endpoint!r} is a network address; the NVLink push is "
                                   f"node-local: use ipc:///path or a filesystem socket path")


def validate_peer_access(prefill_gpus: Iterable[int], decode_gpus: Iterable[int],
                         can_access: Callable[[int, int], bool] | None = None) -> None:
    if can_access is None:
        from infera_b200.ops import _native

        lib = _native.kernels()

        def can_access(a, b):
            return bool(lib.ib_can_access_peer(a, b))

    bad = [(p, d) for p in prefill_gpus for d in decode_gpus if p != d and not can_access(p, d)]
    if bad:
        raise DisaggPreflightError(f"no peer access between prefill and decode GPUs {bad}: the NVLink KV push "
                                   f"needs every pair on one NVLink / NVSwitch domain")


def preflight(*, mode: str, advertise_host: str | None, kv_endpoint: str | None, single_node: bool = True,
              prefill_gpus: Iterable[int] = (), decode_gpus: Iterable[int] = (),
              can_access: Callable[[int, int], bool] | None = None) -> None:
    is_disagg = mode in ("prefill", "decode")
    validate_advertise_host(advertise_host, is_disagg=is_disagg, single_node=single_node)
    validate_kv_endpoint(kv_endpoint, mode=mode)
    pg, dg = list(prefill_gpus), list(decode_gpus)
    if is_disagg and pg and dg:
        validate_peer_access(pg, dg, can_access)

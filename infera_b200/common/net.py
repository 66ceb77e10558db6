"""Port selection that stays clear of the Kubernetes NodePort range.

A worker that picks an ephemeral port inside 30000-32767 can collide with a
NodePort Service opened later on the node; these helpers bind-probe ports
below that range (``infera/common/net.py:124-163`` has the same rule).
"""

from __future__ import annotations

import random
import socket

NODEPORT_LO, NODEPORT_HI = 30000, 32767
DEFAULT_LO, DEFAULT_HI = 20000, 29999


def _free(port: int, host: str) -> bool:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        try:
            s.bind((host, port))
        except OSError:
            return False
    return True


def in_nodeport_range(port: int) -> bool:
    return NODEPORT_LO <= port <= NODEPORT_HI


def free_tcp_port(host: str = "127.0.0.1", lo: int = DEFAULT_LO, hi: int = DEFAULT_HI, tries: int = 200) -> int:
    rng = random.Random()
    for _ in range(tries):
        p = rng.randint(lo, hi)
        if not in_nodeport_range(p) and _free(p, host):
            return p
    raise RuntimeError(f"no free TCP port in [{lo}, {hi}]")


def free_tcp_port_block(n: int, host: str = "127.0.0.1", lo: int = DEFAULT_LO, hi: int = DEFAULT_HI,
                        tries: int = 200) -> int:
    """First port of ``n`` consecutive free ports (e.g. one per DP rank)."""
    rng = random.Random()
    for _ in range(tries):
        base = rng.randint(lo, hi - n + 1)
        ports = range(base, base + n)
        if any(in_nodeport_range(p) for p in ports):
            continue
        if all(_free(p, host) for p in ports):
            return base
    raise RuntimeError(f"no block of {n} free TCP ports in [{lo}, {hi}]")

"""Endpoint picking for a Gateway API Inference Extension (GAIE) gateway.

The gateway forwards the request itself; the endpoint picker only decides
where: the same pool, policy and PD preference as the router's auto mode
(a prefill + decode pair when the model has both pools, else a mixed
worker). The decision is a destination ``host:port`` plus the headers the
worker side needs (``x-worker-instance-id``, ``x-prefill-instance-id``
for the direct-mode router next to the worker). ``release`` returns the
policy's in-flight block references when the request ends.
Role of ``infera/gaie/endpoint_picker.py:29-128``.
"""

from __future__ import annotations

from dataclasses import dataclass
from urllib.parse import urlparse

from infera_b200.common.worker_pool import DisaggMode

DEST_HEADER = "x-gateway-destination-endpoint"
WORKER_HEADER = "x-worker-instance-id"
PREFILL_HEADER = "x-prefill-instance-id"


@dataclass
class PickResult:
    destination: str
    worker_id: str
    prefill_id: str | None
    route_key: str
    blocks: list
    prefill_route_key: str | None = None
    prefill_blocks: list | None = None

    def headers(self) -> dict[str, str]:
        h = {DEST_HEADER: self.destination, WORKER_HEADER: self.worker_id}
        if self.prefill_id:
            h[PREFILL_HEADER] = self.prefill_id
        return h


def endpoint_of(url: str, port_override: int | None = None) -> str:
    u = urlparse(url if "://" in url else f"//{url}")
    if u.hostname and port_override:
        return f"{u.hostname}:{port_override}"
    if u.hostname and u.port:
        return f"{u.hostname}:{u.port}"
    return u.hostname or url


class EndpointPicker:
    def __init__(self, pool, policy, target_port: int | None = None, breaker=None):
        self.pool = pool
        self.policy = policy
        self.target_port = target_port
        self.breaker = breaker

    def _filter(self, ws):
        return self.breaker.filter(ws) if self.breaker is not None else ws

    def pick(self, model: str | None, body: dict) -> PickResult | None:
        pre = self._filter(self.pool.list_active(model=model, mode=DisaggMode.PREFILL))
        dec = self._filter(self.pool.list_active(model=model, mode=DisaggMode.DECODE))
        if pre and dec:
            pt, pb = self.policy.pick(pre, body, role_hint="prefill")
            dt, db = self.policy.pick(dec, body, role_hint="decode")
            self.policy.on_request_started(pt.route_key, pb)
            self.policy.on_request_started(dt.route_key, db)
            return PickResult(endpoint_of(dt.worker.url, self.target_port), dt.worker.worker_id,
                              pt.worker.worker_id, dt.route_key, list(db), pt.route_key, list(pb))
        mixed = self._filter(self.pool.list_active(model=model, mode=DisaggMode.MIXED))
        if not mixed:
            return None
        t, blocks = self.policy.pick(mixed, body)
        self.policy.on_request_started(t.route_key, blocks)
        return PickResult(endpoint_of(t.worker.url, self.target_port), t.worker.worker_id, None, t.route_key,
                          list(blocks))

    def release(self, r: PickResult) -> None:
        self.policy.on_request_finished(r.route_key, r.blocks)
        if r.prefill_route_key:
            self.policy.on_request_finished(r.prefill_route_key, r.prefill_blocks or [])

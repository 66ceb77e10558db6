"""Prometheus metrics of the front door and router.

Metric names follow the reference's ``infera_*`` surface
(``infera/server/metrics.py:41-202``) so dashboards carry over. A dedicated
registry per :class:`RouterMetrics` keeps tests independent.
"""

from __future__ import annotations

import time
from contextlib import contextmanager

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest

CACHE_HIT_BUCKETS = (0.0, 0.1, 0.25, 0.5, 0.75, 0.9, 0.95, 0.99, 1.0)


class RouterMetrics:
    def __init__(self, registry: CollectorRegistry | None = None):
        r = self.registry = registry or CollectorRegistry()
        self.picks = Counter("infera_router_picks_total", "Routing decisions", ["role", "worker_id"], registry=r)
        self.cache_hit_ratio = Histogram("infera_router_cache_hit_ratio", "Prefix-block hit ratio of picks",
                                         ["role"], buckets=CACHE_HIT_BUCKETS, registry=r)
        self.request_blocks = Histogram("infera_router_request_blocks", "Blocks per routed request", ["role"],
                                        buckets=(1, 4, 16, 64, 256, 1024, 4096), registry=r)
        self.requests = Counter("infera_requests_total", "Requests by router and outcome", ["router", "outcome"],
                                registry=r)
        self.duration = Histogram("infera_request_duration_seconds", "End-to-end request duration", ["router"],
                                  registry=r)
        self.inflight = Gauge("infera_requests_inflight", "Requests in flight", ["router"], registry=r)
        self.pd_leg_hist = Histogram("infera_pd_dispatch_duration_seconds", "Per-leg PD dispatch duration", ["leg"],
                                registry=r)
        self.migrations_total = Counter("infera_migrations_total", "Mid-stream migrations", ["reason"], registry=r)
        self.migrations_failed = Counter("infera_migrations_failed_total", "Migrations not possible", ["reason"],
                                         registry=r)
        self.pd_bootstrap_failures = Counter("infera_pd_bootstrap_failures_total", "PD pair failures", ["leg"],
                                             registry=r)
        self.active_workers = Gauge("infera_active_workers", "Workers by status and mode",
                                    ["model", "mode", "status"], registry=r)
        self.breaker_state = Gauge("infera_worker_breaker_state", "0 closed, 1 half-open, 2 open", ["worker_id"],
                                   registry=r)
        self.breaker_trips = Counter("infera_worker_breaker_trips_total", "Breaker trips", ["worker_id"], registry=r)
        self.policy_active_blocks = Gauge("infera_policy_active_blocks", "Distinct in-flight blocks per target",
                                          ["worker_id"], registry=r)
        self.cache_view_size = Gauge("infera_router_cache_view_blocks", "Blocks in the router's view of a worker",
                                     ["worker_id"], registry=r)
        self.cache_control_seen = Counter("infera_cache_control_seen_total", "Retention hints seen",
                                          ["retention"], registry=r)
        self.locality_skipped = Counter("infera_cache_locality_skipped_total", "Picks ignoring locality",
                                        ["reason"], registry=r)

    # ------------------------------------------------------------------ hooks
    def record_pick(self, role: str, worker_id: str, hits: int, blocks: int) -> None:
        self.picks.labels(role=role, worker_id=worker_id).inc()
        if blocks > 0:
            self.cache_hit_ratio.labels(role=role).observe(hits / blocks)
            self.request_blocks.labels(role=role).observe(blocks)

    def set_active_blocks(self, worker_id: str, n: int) -> None:
        self.policy_active_blocks.labels(worker_id=worker_id).set(n)

    def pd_leg(self, leg: str, seconds: float) -> None:
        self.pd_leg_hist.labels(leg=leg).observe(seconds)

    def migrations(self, reason: str) -> None:
        self.migrations_total.labels(reason=reason).inc()

    def breaker_changed(self, worker_id: str, state, tripped: bool) -> None:
        from infera_b200.router.breaker import STATE_VALUE

        self.breaker_state.labels(worker_id=worker_id).set(STATE_VALUE[state.value])
        if tripped:
            self.breaker_trips.labels(worker_id=worker_id).inc()

    @contextmanager
    def track_request(self, router: str):
        obs = {"outcome": "ok"}
        self.inflight.labels(router=router).inc()
        t0 = time.monotonic()
        try:
            yield obs
        except Exception:
            obs["outcome"] = "error"
            raise
        finally:
            self.inflight.labels(router=router).dec()
            self.duration.labels(router=router).observe(time.monotonic() - t0)
            self.requests.labels(router=router, outcome=obs["outcome"]).inc()

    def snapshot_pool(self, pool, kv_client=None) -> None:
        self.active_workers.clear()
        counts: dict[tuple, int] = {}
        for w in pool.all():
            k = (w.model_name, w.disagg_mode.value, w.status.value)
            counts[k] = counts.get(k, 0) + 1
        for (m, mode, st), n in counts.items():
            self.active_workers.labels(model=m, mode=mode, status=st).set(n)
        if kv_client is not None:
            for wid, wv in getattr(kv_client, "workers", {}).items():
                self.cache_view_size.labels(worker_id=wid).set(sum(len(v) for v in wv.views.values()))

    def render(self) -> bytes:
        return generate_latest(self.registry)


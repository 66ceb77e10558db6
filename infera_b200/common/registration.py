"""Worker-side self-registration.

:class:`EtcdRegistration`: grant a lease (TTL 30 s), PUT the record under
``/infera/workers/<host:port>`` with that lease, keep the lease alive every
TTL/3 and re-register when it was lost, revoke it on deregister (the
lifecycle of ``infera/common/registration.py:55-186``). The record carries
identity only; its presence is what makes the worker routable.
"""

from __future__ import annotations

import asyncio
import json
import logging

import httpx

from infera_b200.common.discovery import DEFAULT_PREFIX, b64, normalize_endpoint

logger = logging.getLogger(__name__)

DEFAULT_LEASE_TTL = 30


class EtcdRegistration:
    def __init__(self, endpoint: str, payload: dict, prefix: str = DEFAULT_PREFIX, lease_ttl: int = DEFAULT_LEASE_TTL):
        self.base = normalize_endpoint(endpoint)
        self.payload = payload
        self.key = prefix + payload["worker_id"]
        self.ttl = lease_ttl
        self.lease_id: int | None = None
        self._http = httpx.AsyncClient(base_url=self.base, timeout=10.0)
        self.reregistrations = 0

    async def register(self) -> None:
        r = await self._http.post("/v3/lease/grant", json={"TTL": self.ttl})
        r.raise_for_status()
        self.lease_id = int(r.json()["ID"])
        r = await self._http.post("/v3/kv/put", json={"key": b64(self.key), "value": b64(json.dumps(self.payload)),
                                                      "lease": str(self.lease_id)})
        r.raise_for_status()

    async def keepalive_once(self) -> bool:
        """One keepalive; re-registers if the lease is gone. True if alive."""
        if self.lease_id is None:
            await self.register()
            return True
        r = await self._http.post("/v3/lease/keepalive", json={"ID": str(self.lease_id)})
        r.raise_for_status()
        data = r.json()
        data = data.get("result", data)
        if int(data.get("TTL", 0)) <= 0:
            logger.warning("lease %s lost; re-registering", self.lease_id)
            self.reregistrations += 1
            await self.register()
            return False
        return True

    async def heartbeat_loop(self, interval: float | None = None) -> None:
        interval = interval if interval is not None else max(1.0, self.ttl / 3)
        while True:
            await asyncio.sleep(interval)
            try:
                await self.keepalive_once()
            except asyncio.CancelledError:
                raise
            except Exception as e:
                logger.warning("heartbeat failed: %s", e)

    async def deregister(self) -> None:
        if self.lease_id is not None:
            try:
                await self._http.post("/v3/lease/revoke", json={"ID": str(self.lease_id)})
            except Exception as e:
                logger.warning("lease revoke failed: %s", e)
            self.lease_id = None

    async def close(self) -> None:
        await self._http.aclose()


class InProcessRegistration:
    """Registration against an :class:`InProcessRegistry`."""

    def __init__(self, registry, payload: dict):
        self.registry = registry
        self.payload = payload

    async def register(self) -> None:
        self.registry.register(self.payload)

    async def heartbeat_loop(self, interval: float | None = None) -> None:
        while True:
            await asyncio.sleep(3600)

    async def deregister(self) -> None:
        self.registry.deregister(self.payload["worker_id"])

    async def close(self) -> None:
        return None

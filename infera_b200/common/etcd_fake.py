"""A small in-memory server speaking the etcd v3 HTTP/JSON gateway subset the
registry and registration use: kv range / put / deleterange, lease grant /
keepalive / revoke / expiry, and streaming watch.

There is no etcd binary in this environment; this stands in for it in tests
and single-box deployments (``python -m infera_b200.common.etcd_fake``).
Keys and values are base64 in JSON, revisions are decimal strings, PUT
events carry no ``type`` field (as the real gateway emits them).
"""

from __future__ import annotations

import argparse
import asyncio
import base64
import json
import threading
import time
from dataclasses import dataclass, field

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse


def _b64d(s: str | None) -> bytes:
    return base64.b64decode(s) if s else b""


def _b64e(b: bytes) -> str:
    return base64.b64encode(b).decode()


@dataclass
class _KV:
    value: bytes
    create_rev: int
    mod_rev: int
    version: int
    lease: int


@dataclass
class _Lease:
    ttl: int
    expires: float
    keys: set = field(default_factory=set)


class EtcdState:
    def __init__(self) -> None:
        self.rev = 1
        self.kvs: dict[bytes, _KV] = {}
        self.leases: dict[int, _Lease] = {}
        self.next_lease = 7587000000000000000
        self.watchers: list[tuple[bytes, bytes, asyncio.Queue, asyncio.AbstractEventLoop]] = []
        self.lock = threading.RLock()
        # (revision, event) history, so a watch can start from a past revision
        self.history: list[tuple[int, dict]] = []
        self.history_cap = 100000

    # --------------------------------------------------------------- helpers
    @staticmethod
    def _in_range(k: bytes, key: bytes, end: bytes) -> bool:
        if not end:
            return k == key
        if end == b"\x00":
            return k >= key
        return key <= k < end

    def _notify(self, events: list[dict]) -> None:
        for e in events:
            self.history.append((self.rev, e))
        if len(self.history) > self.history_cap:
            del self.history[: len(self.history) - self.history_cap]
        for key, end, q, loop in list(self.watchers):
            evs = [e for e in events if self._in_range(_b64d(e["kv"]["key"]), key, end)]
            if evs:
                loop.call_soon_threadsafe(q.put_nowait, {"result": {"header": self.header(), "events": evs}})

    def header(self) -> dict:
        return {"cluster_id": "1", "member_id": "1", "revision": str(self.rev), "raft_term": "1"}

    def _kv_json(self, k: bytes, v: _KV) -> dict:
        return {"key": _b64e(k), "value": _b64e(v.value), "create_revision": str(v.create_rev),
                "mod_revision": str(v.mod_rev), "version": str(v.version), "lease": str(v.lease)}

    # --------------------------------------------------------------- ops
    def put(self, key: bytes, value: bytes, lease: int = 0) -> None:
        with self.lock:
            if lease and lease not in self.leases:
                raise KeyError("requested lease not found")
            self.rev += 1
            old = self.kvs.get(key)
            if old is not None and old.lease and old.lease in self.leases:
                self.leases[old.lease].keys.discard(key)
            kv = _KV(value, old.create_rev if old else self.rev, self.rev, (old.version + 1) if old else 1, lease)
            self.kvs[key] = kv
            if lease:
                self.leases[lease].keys.add(key)
            self._notify([{"kv": self._kv_json(key, kv)}])

    def delete(self, key: bytes, end: bytes = b"") -> int:
        with self.lock:
            victims = [k for k in self.kvs if self._in_range(k, key, end)]
            if not victims:
                return 0
            self.rev += 1
            evs = []
            for k in victims:
                kv = self.kvs.pop(k)
                if kv.lease in self.leases:
                    self.leases[kv.lease].keys.discard(k)
                evs.append({"type": "DELETE", "kv": {"key": _b64e(k), "mod_revision": str(self.rev)}})
            self._notify(evs)
            return len(victims)

    def range(self, key: bytes, end: bytes) -> list[tuple[bytes, _KV]]:
        with self.lock:
            return sorted((k, v) for k, v in self.kvs.items() if self._in_range(k, key, end))

    def grant(self, ttl: int) -> int:
        with self.lock:
            self.next_lease += 1
            self.leases[self.next_lease] = _Lease(ttl, time.monotonic() + ttl)
            return self.next_lease

    def keepalive(self, lease: int) -> int:
        with self.lock:
            le = self.leases.get(lease)
            if le is None:
                return 0
            le.expires = time.monotonic() + le.ttl
            return le.ttl

    def revoke(self, lease: int) -> None:
        with self.lock:
            le = self.leases.pop(lease, None)
            if le is not None:
                for k in list(le.keys):
                    self.delete(k)

    def expire(self, now: float | None = None) -> list[int]:
        """Revoke every lease past its TTL (the test hook for lease loss)."""
        now = time.monotonic() if now is None else now
        with self.lock:
            dead = [i for i, le in self.leases.items() if le.expires <= now]
        for i in dead:
            self.revoke(i)
        return dead


def build_app(state: EtcdState | None = None) -> FastAPI:
    st = state or EtcdState()
    app = FastAPI()
    app.state.etcd = st

    @app.get("/health")
    async def health():
        return {"health": "true"}

    @app.post("/v3/kv/range")
    async def kv_range(req: Request):
        body = await req.json()
        items = st.range(_b64d(body.get("key")), _b64d(body.get("range_end")))
        kvs = [st._kv_json(k, v) for k, v in items]
        out = {"header": st.header(), "count": str(len(kvs))}
        if kvs:
            out["kvs"] = kvs
        return out

    @app.post("/v3/kv/put")
    async def kv_put(req: Request):
        body = await req.json()
        try:
            st.put(_b64d(body.get("key")), _b64d(body.get("value")), int(body.get("lease", 0) or 0))
        except KeyError as e:
            return JSONResponse({"error": str(e), "code": 5, "message": str(e)}, status_code=400)
        return {"header": st.header()}

    @app.post("/v3/kv/deleterange")
    async def kv_del(req: Request):
        body = await req.json()
        n = st.delete(_b64d(body.get("key")), _b64d(body.get("range_end")))
        return {"header": st.header(), "deleted": str(n)}

    @app.post("/v3/lease/grant")
    async def lease_grant(req: Request):
        body = await req.json()
        ttl = int(body.get("TTL", 30))
        return {"header": st.header(), "ID": str(st.grant(ttl)), "TTL": str(ttl)}

    @app.post("/v3/lease/keepalive")
    async def lease_keepalive(req: Request):
        body = await req.json()
        lid = int(body.get("ID", 0))
        ttl = st.keepalive(lid)
        return {"result": {"header": st.header(), "ID": str(lid), "TTL": str(ttl)}}

    @app.post("/v3/lease/revoke")
    async def lease_revoke(req: Request):
        body = await req.json()
        st.revoke(int(body.get("ID", 0)))
        return {"header": st.header()}

    @app.post("/v3/watch")
    async def watch(req: Request):
        body = await req.json()
        cr = body.get("create_request", {})
        key, end = _b64d(cr.get("key")), _b64d(cr.get("range_end"))
        q: asyncio.Queue = asyncio.Queue()
        entry = (key, end, q, asyncio.get_running_loop())
        start = int(cr.get("start_revision", 0) or 0)
        with st.lock:
            # replay what happened since start_revision (as etcd does), then go live
            if start > 0:
                past = [e for rev, e in st.history if rev >= start and st._in_range(_b64d(e["kv"]["key"]), key, end)]
                if past:
                    q.put_nowait({"result": {"header": st.header(), "events": past}})
            st.watchers.append(entry)

        async def gen():
            try:
                yield json.dumps({"result": {"header": st.header(), "created": True}}) + "\n"
                while True:
                    if await req.is_disconnected():
                        return
                    try:
                        msg = await asyncio.wait_for(q.get(), timeout=1.0)
                    except asyncio.TimeoutError:
                        continue
                    yield json.dumps(msg) + "\n"
            finally:
                if entry in st.watchers:
                    st.watchers.remove(entry)

        return StreamingResponse(gen(), media_type="application/json")

    async def expiry_loop():
        while True:
            await asyncio.sleep(0.5)
            st.expire()

    @app.on_event("startup")
    async def _start():
        app.state.expiry = asyncio.create_task(expiry_loop())

    return app


def main(argv=None) -> None:
    import uvicorn

    ap = argparse.ArgumentParser(description="in-memory etcd v3 JSON gateway")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=2379)
    a = ap.parse_args(argv)
    uvicorn.run(build_app(), host=a.host, port=a.port, log_level="warning")


if __name__ == "__main__":
    main()

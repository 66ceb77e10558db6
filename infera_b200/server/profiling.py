"""``POST /v1/admin/profile/{start,stop}`` fan-out.

Selects workers by ``worker_id`` / ``model`` / ``role`` (any omitted field
matches all) and POSTs ``{url}/{action}_profile`` to each concurrently,
returning per-worker results (``infera/server/profiling.py:49-142``). The
engines answer with a torch.profiler trace (NVTX ranges per phase)."""

from __future__ import annotations

import asyncio


def select_targets(pool, worker_id=None, model=None, role=None) -> list:
    out = []
    for w in pool.list_active():
        if worker_id and w.worker_id != worker_id:
            continue
        if model and w.model_name != model:
            continue
        if role and w.disagg_mode.value != role:
            continue
        out.append(w)
    return out


class ProfileFanout:
    def __init__(self, pool, transport):
        self.pool = pool
        self.transport = transport

    async def fan_out(self, action: str, body: dict) -> dict:
        targets = select_targets(self.pool, body.get("worker_id"), body.get("model"), body.get("role"))
        payload = {k: v for k, v in body.items() if k not in ("worker_id", "model", "role")}

        async def one(w):
            try:
                r = await self.transport.post(w, f"/{action}_profile", payload)
                return w.worker_id, {"status": r.status_code, "ok": r.status_code < 400}
            except Exception as e:  # transport failures are reported, not raised
                return w.worker_id, {"status": 0, "ok": False, "error": str(e)}

        res = await asyncio.gather(*(one(w) for w in targets))
        return {"action": action, "targets": [w.worker_id for w in targets], "results": dict(res)}

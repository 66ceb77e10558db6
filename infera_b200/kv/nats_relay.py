"""Worker-side relay of KV events onto NATS.

Tails the engine's local ZMQ KV-event publisher (topic ``kv-events``, one
msgpack batch per message) and republishes every batch unchanged on
``infera.kv.events.<worker token>``, where routers started with
``--kv-event-transport nats`` receive them (``KvEventClient.attach_nats``).

With ``jetstream=True`` the batches go into the JetStream stream
``INFERA_KV_EVENTS`` (acked publishes), and the relay keeps this worker's
routing view - the router-hash set and the engine-hash map it derives from
the events, the same structures the router keeps - in the key-value bucket
``INFERA_KV_VIEWS`` under the worker token, refreshed at most every
``view_period_s`` while it changes: a router that starts (or reconnects)
later bootstraps from the bucket instead of an HTTP snapshot.

Reference counterpart: ``KvEventNatsRelay`` (``infera/kv/nats_relay.py:57``)
with its stream and bucket (``infera/kv/nats_bus.py:33-259``).
"""

from __future__ import annotations

import asyncio
import logging

from infera_b200.router.kv_event.client import NATS_SUBJECT, TOPIC, worker_token

logger = logging.getLogger(__name__)


KV_STREAM = "INFERA_KV_EVENTS"
VIEW_BUCKET = "INFERA_KV_VIEWS"


def encode_view(wv) -> bytes:
    """A worker's routing view (per DP rank: router-hash set + engine-hash ->
    router-hash map) as the bucket value."""
    import msgpack

    return msgpack.packb({"block_size": wv.block_size,
                          "ranks": [[r, sorted(wv.views.get(r, ())), list(wv.maps.get(r, {}).items())]
                                    for r in sorted(set(wv.views) | set(wv.maps), key=lambda x: -1 if x is None else x)]},
                         use_bin_type=True)


def decode_view(raw: bytes) -> dict:
    """{rank: (router-hash set, engine-hash map)} from a bucket value."""
    import msgpack

    d = msgpack.unpackb(raw, raw=False, strict_map_key=False)
    return {r: (set(view), {int(a): int(b) for a, b in hmap}) for r, view, hmap in d.get("ranks", [])}


class KvEventNatsRelay:
    def __init__(self, bus, worker_id: str, zmq_endpoint: str, jetstream: bool = False, block_size: int = 16,
                 engine: str = "infera-b200", view_period_s: float = 1.0):
        self.bus = bus
        self.worker_id = worker_id
        self.token = worker_token(worker_id)
        self.subject = NATS_SUBJECT + self.token
        self.endpoint = zmq_endpoint.replace("tcp://*:", "tcp://127.0.0.1:").replace("tcp://0.0.0.0:",
                                                                                      "tcp://127.0.0.1:")
        self.jetstream = jetstream
        self.view_period_s = view_period_s
        self.relayed = 0
        self.views_put = 0
        self._task: asyncio.Task | None = None
        self._view_task: asyncio.Task | None = None
        self._mirror = None
        self._dirty = False
        if jetstream:
            from infera_b200.router.kv_event.client import KvEventClient, WorkerView

            self._mirror = KvEventClient(use_zmq=False)
            self._mirror.workers[worker_id] = WorkerView(worker_id, int(block_size), engine)

    def start(self) -> None:
        self._task = asyncio.get_running_loop().create_task(self._run())

    async def _run(self) -> None:
        import zmq
        import zmq.asyncio

        sock = zmq.asyncio.Context.instance().socket(zmq.SUB)
        try:
            sock.connect(self.endpoint)
            sock.subscribe(TOPIC)
            js = kv = None
            if self.jetstream:
                from infera_b200.common.jetstream import JetStream

                js = JetStream(self.bus)
                await js.add_stream(KV_STREAM, [NATS_SUBJECT + ">"], max_age_s=600.0)
                kv = await js.key_value(VIEW_BUCKET)
                self._view_task = asyncio.get_running_loop().create_task(self._views(kv))
            while True:
                frames = await sock.recv_multipart()
                await self.relay(frames[-1], js)
        except asyncio.CancelledError:
            pass
        except Exception as e:   # the worker keeps serving; the router falls back to snapshots
            logger.warning("kv event relay stopped: %s", e)
        finally:
            sock.close(linger=0)

    async def relay(self, raw: bytes, js=None) -> None:
        """Republish one batch (and fold it into the bucket's view)."""
        if js is not None:
            await js.publish(self.subject, raw)
            self._fold(raw)
        else:
            await self.bus.publish(self.subject, raw)
        self.relayed += 1

    def _fold(self, raw: bytes) -> None:
        from infera_b200.router.kv_event.events import decoder_for_engine

        wv = self._mirror.workers[self.worker_id]
        batch = decoder_for_engine(wv.engine).decode(raw)
        for ev in batch.events:
            self._mirror._handle(wv, ev, batch.attn_dp_rank)
        self._dirty = True

    async def _views(self, kv) -> None:
        while True:
            await asyncio.sleep(self.view_period_s)
            if self._dirty:
                self._dirty = False
                await kv.put(self.token, encode_view(self._mirror.workers[self.worker_id]))
                self.views_put += 1

    async def flush_view(self, kv) -> None:
        if self._mirror is not None:
            await kv.put(self.token, encode_view(self._mirror.workers[self.worker_id]))
            self.views_put += 1

    async def stop(self) -> None:
        if self._view_task is not None:
            self._view_task.cancel()
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass

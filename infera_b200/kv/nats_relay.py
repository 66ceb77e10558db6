"""Worker-side relay of KV events onto NATS.

Tails the engine's local ZMQ KV-event publisher (topic ``kv-events``, one
msgpack batch per message) and republishes every batch unchanged on
``infera.kv.events.<worker token>``, where routers started with
``--kv-event-transport nats`` receive them (``KvEventClient.attach_nats``).
A router that starts later rebuilds its view from the worker's snapshot
endpoint, as on the ZMQ path.

Reference counterpart: ``KvEventNatsRelay`` (``infera/kv/nats_relay.py:57``),
which republishes into a JetStream stream and keeps a KV-bucket snapshot;
here the bus is core NATS and the snapshot stays on HTTP.
"""

from __future__ import annotations

import asyncio
import logging

from infera_b200.router.kv_event.client import NATS_SUBJECT, TOPIC, worker_token

logger = logging.getLogger(__name__)


class KvEventNatsRelay:
    def __init__(self, bus, worker_id: str, zmq_endpoint: str):
        self.bus = bus
        self.subject = NATS_SUBJECT + worker_token(worker_id)
        self.endpoint = zmq_endpoint.replace("tcp://*:", "tcp://127.0.0.1:").replace("tcp://0.0.0.0:",
                                                                                      "tcp://127.0.0.1:")
        self.relayed = 0
        self._task: asyncio.Task | None = None

    def start(self) -> None:
        self._task = asyncio.get_running_loop().create_task(self._run())

    async def _run(self) -> None:
        import zmq
        import zmq.asyncio

        sock = zmq.asyncio.Context.instance().socket(zmq.SUB)
        try:
            sock.connect(self.endpoint)
            sock.subscribe(TOPIC)
            while True:
                frames = await sock.recv_multipart()
                await self.bus.publish(self.subject, frames[-1])
                self.relayed += 1
        except asyncio.CancelledError:
            pass
        except Exception as e:   # the worker keeps serving; the router falls back to snapshots
            logger.warning("kv event relay stopped: %s", e)
        finally:
            sock.close(linger=0)

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass

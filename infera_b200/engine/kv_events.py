"""Engine-side KV-event publisher.

Collects the block manager's (kind, payload) callbacks into
``KVEventBatch`` messages (vLLM map encoding) and publishes them on a ZMQ
PUB socket as multipart ``[topic, seq (u64 BE), msgpack batch]``, flushing
at most every ``flush_ms`` or when ``max_events`` are pending. In-process
sinks (the router's client in tests and single-process fleets) can be
attached with :meth:`add_sink`.
"""

from __future__ import annotations

import threading
import time

from infera_b200.router.kv_event.events import KVEventBatch, encode_batch, event_from_dict

TOPIC = b"kv-events"


class KvEventPublisher:
    def __init__(self, endpoint: str | None = None, dp_rank: int | None = None, flush_ms: float = 5.0,
                 max_events: int = 256):
        self.endpoint = endpoint
        self.dp_rank = dp_rank
        self.flush_s = flush_ms / 1000.0
        self.max_events = max_events
        self._pending: list = []
        self._lock = threading.Lock()
        self._seq = 0
        self._last = time.monotonic()
        self._sock = None
        self._sinks: list = []
        self.published = 0
        if endpoint:
            import zmq

            ctx = zmq.Context.instance()
            self._sock = ctx.socket(zmq.PUB)
            self._sock.setsockopt(zmq.SNDHWM, 100000)
            self._sock.bind(endpoint)

    def add_sink(self, fn) -> None:
        """fn(events: list) is called with each flushed batch's events."""
        self._sinks.append(fn)

    def __call__(self, kind: str, payload: dict) -> None:
        ev = event_from_dict(kind, payload)
        with self._lock:
            self._pending.append(ev)
            n = len(self._pending)
        if n >= self.max_events or time.monotonic() - self._last >= self.flush_s:
            self.flush()

    def flush(self) -> None:
        with self._lock:
            if not self._pending:
                self._last = time.monotonic()
                return
            evs, self._pending = self._pending, []
            self._last = time.monotonic()
            seq = self._seq
            self._seq += 1
        batch = KVEventBatch(ts=time.time(), events=evs, attn_dp_rank=self.dp_rank)
        if self._sock is not None:
            self._sock.send_multipart([TOPIC, seq.to_bytes(8, "big"), encode_batch(batch)])
        for fn in self._sinks:
            fn(evs)
        self.published += len(evs)

    def close(self) -> None:
        self.flush()
        if self._sock is not None:
            self._sock.close(linger=0)
            self._sock = None

"""Publisher side of the tier-aware KV index: ZMQ PUB of ``EventBatch`` es
(multipart ``[b"kv-index", seq u64 BE, msgpack]``), batched per probe flush.
Role of ``infera/kv/publisher.py:46``."""

from __future__ import annotations

from infera_b200.kv.wire import TOPIC, EventBatch, encode_batch


class KvIndexPublisher:
    def __init__(self, endpoint: str):
        import zmq

        self._sock = zmq.Context.instance().socket(zmq.PUB)
        self._sock.setsockopt(zmq.SNDHWM, 100000)
        self._sock.bind(endpoint)
        self.seq = 0

    def __call__(self, batch: EventBatch) -> None:
        self._sock.send_multipart([TOPIC, self.seq.to_bytes(8, "big"), encode_batch(batch)])
        self.seq += 1

    def close(self) -> None:
        self._sock.close(linger=0)

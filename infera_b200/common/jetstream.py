"""JetStream (NATS persistence) over :class:`~infera_b200.common.nats_wire.NatsBus`.

The JetStream API is plain request / reply with JSON bodies on
``$JS.API.*`` subjects; this module speaks that subset of it:

* streams: ``STREAM.CREATE`` / ``STREAM.UPDATE`` / ``STREAM.INFO`` (limits or
  work-queue retention, memory or file storage, per-subject message limit);
* publishing with a ``PubAck`` (``{"stream", "seq"}``);
* consumers: durable pull consumers (``CONSUMER.CREATE`` with an explicit ack
  policy, ``CONSUMER.INFO`` for the pending count, ``CONSUMER.MSG.NEXT`` to
  fetch a batch, ``+ACK`` on the message's reply subject) and ephemeral push
  consumers (``deliver_subject``, deliver policy all / new /
  last_per_subject);
* key-value buckets: stream ``KV_<bucket>`` over ``$KV.<bucket>.>`` keeping
  one message per key; ``get`` reads the last message of a key
  (``STREAM.MSG.GET`` with ``last_by_subj``), ``watch`` replays the latest
  value of every key and follows new ones.

Roles of the nats-py JetStream calls the reference makes in
``infera/kv/nats_bus.py:33-259`` (KV-event stream and view bucket) and
``infera/common/nats_request.py:219-368`` (work-queue request stream).
"""

from __future__ import annotations

import base64
import json
from dataclasses import dataclass


class JetStreamError(RuntimeError):
    def __init__(self, code: int, err_code: int, description: str):
        super().__init__(f"JetStream error {code}/{err_code}: {description}")
        self.code, self.err_code, self.description = code, err_code, description


STREAM_NAME_IN_USE = 10058


@dataclass
class JsMsg:
    subject: str
    data: bytes
    headers: dict
    reply: str | None      # $JS.ACK... subject
    seq: int = 0


def _ack_seq(reply: str | None) -> int:
    """Stream sequence of a delivered message from its ack subject
    ``$JS.ACK.<stream>.<consumer>.<delivered>.<stream seq>.<consumer seq>.<ts>.<pending>``."""
    if not reply or not reply.startswith("$JS.ACK."):
        return 0
    parts = reply.split(".")
    try:
        return int(parts[5])
    except (IndexError, ValueError):
        return 0


class JetStream:
    def __init__(self, bus, api_prefix: str = "$JS.API", timeout: float = 5.0):
        self.bus = bus
        self.api = api_prefix
        self.timeout = timeout

    async def _call(self, subject: str, body: dict | None = None) -> dict:
        m = await self.bus.request(f"{self.api}.{subject}", json.dumps(body or {}).encode(), timeout=self.timeout)
        if m.headers.get("status") == "503":
            raise JetStreamError(503, 0, "JetStream not enabled (no responders)")
        d = json.loads(m.data or b"{}")
        err = d.get("error")
        if err:
            raise JetStreamError(int(err.get("code", 0)), int(err.get("err_code", 0)), err.get("description", ""))
        return d

    # ------------------------------------------------------------------ streams
    async def add_stream(self, name: str, subjects: list[str], retention: str = "limits", storage: str = "memory",
                         max_msgs_per_subject: int = -1, max_age_s: float = 0.0, max_bytes: int = -1) -> dict:
        """Create the stream, or bring an existing one to this configuration."""
        cfg = {"name": name, "subjects": subjects, "retention": retention, "storage": storage,
               "max_msgs_per_subject": max_msgs_per_subject, "max_age": int(max_age_s * 1e9),
               "max_bytes": max_bytes, "discard": "old", "num_replicas": 1}
        try:
            return await self._call(f"STREAM.CREATE.{name}", cfg)
        except JetStreamError as e:
            if e.err_code != STREAM_NAME_IN_USE:
                raise
            return await self._call(f"STREAM.UPDATE.{name}", cfg)

    async def stream_info(self, name: str) -> dict:
        return await self._call(f"STREAM.INFO.{name}")

    async def publish(self, subject: str, data: bytes, headers: dict | None = None) -> dict:
        """Publish into the stream that captures ``subject``; returns its
        PubAck ``{"stream", "seq"}``."""
        inbox = self.bus.new_inbox()
        import asyncio

        fut = asyncio.get_running_loop().create_future()

        async def on_ack(m):
            if not fut.done():
                fut.set_result(m)

        unsub = await self.bus.subscribe(inbox, on_ack)
        try:
            await self.bus.publish(subject, data, headers=headers, reply=inbox)
            m = await asyncio.wait_for(fut, self.timeout)
        finally:
            unsub()
        if m.headers.get("status") == "503":
            raise JetStreamError(503, 0, f"no stream captures {subject}")
        d = json.loads(m.data or b"{}")
        if d.get("error"):
            e = d["error"]
            raise JetStreamError(int(e.get("code", 0)), int(e.get("err_code", 0)), e.get("description", ""))
        return d

    async def get_last(self, stream: str, subject: str) -> JsMsg | None:
        """The last message stored for ``subject`` (None if there is none)."""
        try:
            d = await self._call(f"STREAM.MSG.GET.{stream}", {"last_by_subj": subject})
        except JetStreamError as e:
            if e.code == 404:
                return None
            raise
        msg = d["message"]
        hdrs = {}
        if msg.get("hdrs"):
            from infera_b200.common.nats_wire import parse_headers

            hdrs = parse_headers(base64.b64decode(msg["hdrs"]))
        return JsMsg(msg["subject"], base64.b64decode(msg.get("data") or b""), hdrs, None, int(msg.get("seq", 0)))

    # ------------------------------------------------------------------ consumers
    async def add_consumer(self, stream: str, durable: str | None = None, filter_subject: str | None = None,
                           deliver_policy: str = "all", ack_policy: str = "explicit",
                           deliver_subject: str | None = None, max_ack_pending: int = -1) -> dict:
        cfg = {"deliver_policy": deliver_policy, "ack_policy": ack_policy, "max_ack_pending": max_ack_pending}
        if durable:
            cfg["durable_name"] = durable
        if filter_subject:
            cfg["filter_subject"] = filter_subject
        if deliver_subject:
            cfg["deliver_subject"] = deliver_subject
        subj = f"CONSUMER.CREATE.{stream}" + (f".{durable}" if durable else "")
        return await self._call(subj, {"stream_name": stream, "config": cfg})

    async def consumer_info(self, stream: str, durable: str) -> dict:
        return await self._call(f"CONSUMER.INFO.{stream}.{durable}")

    async def fetch(self, stream: str, durable: str, batch: int = 1, expires_s: float = 1.0) -> list[JsMsg]:
        """Pull up to ``batch`` messages from a durable consumer, waiting at
        most ``expires_s`` for the first."""
        import asyncio

        inbox = self.bus.new_inbox()
        got: list[JsMsg] = []
        done = asyncio.Event()

        async def on_msg(m):
            if m.headers.get("status") in ("404", "408", "409"):   # no messages / expired / closed
                done.set()
                return
            got.append(JsMsg(m.subject, m.data, m.headers, m.reply, _ack_seq(m.reply)))
            if len(got) >= batch:
                done.set()

        unsub = await self.bus.subscribe(inbox, on_msg)
        try:
            await self.bus.publish(f"{self.api}.CONSUMER.MSG.NEXT.{stream}.{durable}",
                                   json.dumps({"batch": batch, "expires": int(expires_s * 1e9)}).encode(),
                                   reply=inbox)
            try:
                await asyncio.wait_for(done.wait(), expires_s + 1.0)
            except asyncio.TimeoutError:
                pass
        finally:
            unsub()
        return got

    async def ack(self, msg: JsMsg) -> None:
        if msg.reply:
            await self.bus.publish(msg.reply, b"+ACK")

    async def subscribe_push(self, stream: str, cb, filter_subject: str | None = None,
                             deliver_policy: str = "new"):
        """Ephemeral push consumer: ``cb(JsMsg)`` for each delivered message
        (no acks). Returns the unsubscribe callable."""
        inbox = self.bus.new_inbox()

        async def on_msg(m):
            await cb(JsMsg(m.subject, m.data, m.headers, m.reply, _ack_seq(m.reply)))

        unsub = await self.bus.subscribe(inbox, on_msg)
        await self.add_consumer(stream, filter_subject=filter_subject, deliver_policy=deliver_policy,
                                ack_policy="none", deliver_subject=inbox)
        return unsub

    # ------------------------------------------------------------------ key-value buckets
    async def key_value(self, bucket: str, storage: str = "memory") -> "KeyValue":
        await self.add_stream(f"KV_{bucket}", [f"$KV.{bucket}.>"], storage=storage, max_msgs_per_subject=1)
        return KeyValue(self, bucket)


class KeyValue:
    def __init__(self, js: JetStream, bucket: str):
        self.js, self.bucket = js, bucket
        self.stream = f"KV_{bucket}"

    def _subject(self, key: str) -> str:
        return f"$KV.{self.bucket}.{key}"

    async def put(self, key: str, value: bytes) -> int:
        return int((await self.js.publish(self._subject(key), value))["seq"])

    async def delete(self, key: str) -> int:
        return int((await self.js.publish(self._subject(key), b"", headers={"KV-Operation": "DEL"}))["seq"])

    async def get(self, key: str) -> bytes | None:
        m = await self.js.get_last(self.stream, self._subject(key))
        if m is None or m.headers.get("KV-Operation") in ("DEL", "PURGE"):
            return None
        return m.data

    async def watch(self, cb) -> object:
        """``cb(key, value | None)`` with the latest value of every key, then
        every later change (None: deleted). Returns the unsubscribe callable."""
        prefix = f"$KV.{self.bucket}."

        async def on_msg(m: JsMsg):
            deleted = m.headers.get("KV-Operation") in ("DEL", "PURGE")
            await cb(m.subject[len(prefix):], None if deleted else m.data)

        return await self.js.subscribe_push(self.stream, on_msg, filter_subject=f"{prefix}>",
                                            deliver_policy="last_per_subject")

"""The JetStream client against the protocol stub: streams with PubAcks,
work-queue retention with a durable pull consumer (pending counts, fetch,
ack removes), push consumers replaying the last message per subject then
following new ones, and key-value buckets (put / get / delete / watch)."""

import asyncio

import pytest

from infera_b200.common.jetstream import JetStream, JetStreamError
from infera_b200.common.nats_wire import NatsBus
from tests.nats_stub import Broker


def _run(coro):
    return asyncio.run(coro)


def test_streams_workqueue_pull_and_push():
    async def go():
        br = await Broker().start()
        bus = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        js = JetStream(bus)
        await js.add_stream("REQ", ["req.>"], retention="workqueue")
        await js.add_stream("REQ", ["req.>"], retention="workqueue")     # idempotent (update)
        acks = [await js.publish(f"req.w{i % 2}", f"m{i}".encode(), headers={"inbox": f"x{i}"}) for i in range(5)]
        await js.add_consumer("REQ", durable="w0", filter_subject="req.w0")
        info = await js.consumer_info("REQ", "w0")
        got = await js.fetch("REQ", "w0", batch=2, expires_s=0.5)
        for m in got:
            await js.ack(m)
        await asyncio.sleep(0.05)
        info2 = await js.consumer_info("REQ", "w0")
        st = await js.stream_info("REQ")
        # a pull that waits for a message published later
        fut = asyncio.ensure_future(js.fetch("REQ", "w0", batch=1, expires_s=2.0))
        await asyncio.sleep(0.1)
        await js.publish("req.w0", b"late")
        late = await fut
        empty = await js.fetch("REQ", "w0", batch=1, expires_s=0.2)
        # push consumer: last message per subject, then new ones
        await js.add_stream("EV", ["ev.>"], max_msgs_per_subject=-1)
        for i in range(3):
            await js.publish("ev.a", f"a{i}".encode())
        await js.publish("ev.b", b"b0")
        seen = []

        async def cb(m):
            seen.append((m.subject, m.data))

        unsub = await js.subscribe_push("EV", cb, filter_subject="ev.>", deliver_policy="last_per_subject")
        await js.publish("ev.a", b"a3")
        await asyncio.sleep(0.1)
        unsub()
        with pytest.raises(JetStreamError):
            await js.publish("nostream.x", b"x")
        await bus.close()
        await br.stop()
        return acks, info, got, info2, st, late, empty, seen

    acks, info, got, info2, st, late, empty, seen = _run(go())
    assert [a["seq"] for a in acks] == [1, 2, 3, 4, 5] and acks[0]["stream"] == "REQ"
    assert info["num_pending"] == 3
    assert [m.data for m in got] == [b"m0", b"m2"] and got[0].headers.get("inbox") == "x0" and got[1].seq == 3
    assert info2["num_pending"] == 1 and info2["num_ack_pending"] == 0
    assert st["state"]["messages"] == 3                      # acked work-queue messages are gone
    assert [m.data for m in late] == [b"m4"]                   # the oldest pending one first
    assert [m.data for m in empty] == [b"late"]
    assert seen == [("ev.a", b"a2"), ("ev.b", b"b0"), ("ev.a", b"a3")]


def test_key_value_bucket():
    async def go():
        br = await Broker().start()
        bus = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        js = JetStream(bus)
        kv = await js.key_value("VIEWS")
        await kv.put("w1", b"v1")
        await kv.put("w1", b"v2")
        await kv.put("w2", b"x")
        got = (await kv.get("w1"), await kv.get("w2"), await kv.get("nope"))
        seen = []

        async def cb(k, v):
            seen.append((k, v))

        unsub = await kv.watch(cb)
        await kv.delete("w2")
        await kv.put("w3", b"z")
        await asyncio.sleep(0.1)
        unsub()
        after = await kv.get("w2")
        await bus.close()
        await br.stop()
        return got, seen, after

    got, seen, after = _run(go())
    assert got == (b"v2", b"x", None)
    assert seen == [("w1", b"v2"), ("w2", b"x"), ("w2", None), ("w3", b"z")]
    assert after is None


def test_kv_events_over_jetstream_with_bucket_bootstrap():
    """A worker's relay puts its KV-event batches into the stream and its
    routing view into the bucket; a router that attaches later bootstraps
    the view from the bucket, then follows new batches from the stream."""
    import time as _time

    from infera_b200.common.worker_pool import WorkerInfo
    from infera_b200.kv.nats_relay import VIEW_BUCKET, KvEventNatsRelay
    from infera_b200.router.kv_event.client import KvEventClient
    from infera_b200.router.kv_event.events import KVEventBatch, encode_batch, event_from_dict
    from infera_b200.utils.hashing import chain_hashes

    a = list(range(100, 164))          # 4 blocks of 16
    b = list(range(500, 532))          # 2 blocks

    def stored(tokens, engine_hashes, parent=None):
        ev = event_from_dict("BlockStored", {"block_hashes": engine_hashes, "parent_block_hash": parent,
                                             "token_ids": tokens, "block_size": 16, "lora_id": None,
                                             "medium": "GPU"})
        return encode_batch(KVEventBatch(ts=_time.time(), events=[ev], attn_dp_rank=None))

    def removed(engine_hashes):
        ev = event_from_dict("BlockRemoved", {"block_hashes": engine_hashes, "medium": "GPU"})
        return encode_batch(KVEventBatch(ts=_time.time(), events=[ev], attn_dp_rank=None))

    async def go():
        br = await Broker().start()
        bw = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        brt = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        wid = "10.0.0.1:9000"
        relay = KvEventNatsRelay(bw, wid, "tcp://127.0.0.1:1", jetstream=True, block_size=16)
        js = JetStream(bw)
        await js.add_stream("INFERA_KV_EVENTS", ["infera.kv.events.>"], max_age_s=600.0)
        kv = await js.key_value(VIEW_BUCKET)
        await relay.relay(stored(a, [11, 12, 13, 14]), js)       # before any router exists
        await relay.flush_view(kv)
        client = KvEventClient(use_zmq=False)
        client.on_worker_added(WorkerInfo(worker_id=wid, url="http://x", model_name="m", kv_block_size=16))
        await client.attach_nats(brt, jetstream=True)
        await asyncio.sleep(0.1)
        boot = set(client.cache_view(wid))
        await relay.relay(stored(b, [21, 22]), js)
        await relay.relay(removed([14]), js)
        await asyncio.sleep(0.1)
        live = set(client.cache_view(wid))
        await client.aclose()
        await bw.close()
        await brt.close()
        await br.stop()
        return boot, live, client.stats

    boot, live, stats = _run(go())
    ha, hb = chain_hashes(a, 16), chain_hashes(b, 16)
    assert boot == set(ha) and stats.get("bootstraps", 0) >= 1
    assert live == set(ha[:3]) | set(hb)


def test_bus_requests_through_the_workqueue():
    """jetstream=True: the router publishes into the INFERA_REQUESTS work
    queue (inbox in a header), the worker pulls from its durable consumer;
    admission follows the consumer's pending count."""
    from infera_b200.common.request_transport import BusRequestClient, BusRequestServer
    from infera_b200.common.worker_pool import WorkerInfo
    from infera_b200.router.transport import DATA, DONE

    async def handler(path, body, headers):
        for i in range(body.get("n", 2)):
            yield DATA, 200, f"t{i}".encode()
        yield DONE, 200, b""

    async def go():
        br = await Broker().start()
        bw = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        brt = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        w = WorkerInfo(worker_id="10.0.0.2:9000", url="bus://", model_name="m")
        cli = BusRequestClient(brt, jetstream=True, max_pending=2)
        before = await cli.admit(w)                                   # no consumer yet: not admitted
        srv = BusRequestServer(bw, BusRequestClient.token(w), handler, jetstream=True)
        await srv.start()
        frames = [x async for x in cli.stream(w, "/v1/completions", {"n": 3})]
        js = await cli._jetstream()
        # a backlog at the limit refuses admission (worker stopped pulling;
        # its last pull request expires first)
        await srv.stop()
        await asyncio.sleep(1.3)
        for _ in range(2):
            await js.publish("infera.req." + BusRequestClient.token(w), b"{}", headers={"rid": "x"})
        full = await cli.admit(w)
        await bw.close()
        await brt.close()
        await br.stop()
        return before, frames, full, srv.stats

    before, frames, full, stats = _run(go())
    assert before is False
    assert [f[2] for f in frames] == [b"t0", b"t1", b"t2", b""] and frames[-1][0] == "done"
    assert full is False and stats["served"] == 1

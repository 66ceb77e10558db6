"""Control-plane pieces on CPU: engine metrics parsing, HTTP drain, ports,
log scrubbing, PD preflight, Kubernetes discovery / registration against a
fake API server, and the bus request transport (admission, cancel on idle
timeout, drain with hand-back)."""

import asyncio
import json

import pytest

from infera_b200.common import engine_metrics as em
from infera_b200.common.disagg_preflight import DisaggPreflightError, preflight
from infera_b200.common.discovery_k8s import WORKER_INFO_ANNOTATION, KubernetesRegistry
from infera_b200.common.k8s_client import FakeK8sClient, merge_patch
from infera_b200.common.logsafe import scrub
from infera_b200.common.net import free_tcp_port, free_tcp_port_block, in_nodeport_range
from infera_b200.common.registration_k8s import K8sRegistration
from infera_b200.common.request_transport import BusRequestClient, BusRequestServer, InProcessBus
from infera_b200.common.worker_pool import EngineType, WorkerInfo, WorkerStatus
from infera_b200.engine.drain import drain_engine_inflight
from infera_b200.router.transport import DATA, DONE, DRAINING_NOTICE, ERROR

SGL = """# HELP sglang:num_running_reqs x
sglang:num_running_reqs{tp_rank="0"} 2
sglang:num_running_reqs{tp_rank="1"} 0
sglang:num_queue_reqs{tp_rank="0"} 1
sglang:num_prefill_inflight_queue_reqs 3
"""


def test_engine_metrics():
    assert em.inflight_from_metrics(SGL, EngineType.SGLANG) == 6.0
    assert em.inflight_from_metrics(SGL, EngineType.SGLANG, draining=False) == 3.0
    assert em.inflight_from_metrics("vllm:num_requests_running 1\n", EngineType.VLLM) is None  # waiting missing
    v = "vllm:num_requests_running 0\nvllm:num_requests_waiting 0\nvllm:gpu_cache_usage_perc 0.5\n"
    assert em.inflight_from_metrics(v, "vllm") == 0.0
    assert em.read_gauge(v, "kv_cache_usage", EngineType.VLLM) == 0.5


def test_http_drain_settle_and_unknown():
    clock = [0.0]
    seq = iter([2, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0])

    async def fetch():
        n = next(seq)
        return f"infera_engine:num_requests_running {n}\ninfera_engine:num_requests_waiting 0\n"

    async def sleep(dt):
        clock[0] += dt

    res = asyncio.run(drain_engine_inflight(fetch, "infera-b200", timeout=30, settle_s=2.0, poll_s=0.5,
                                            clock=lambda: clock[0], sleep=sleep))
    assert res["drained"] and res["waited_s"] >= 2.0

    async def missing():
        return "something_else 1\n"

    res = asyncio.run(drain_engine_inflight(missing, "vllm", sleep=sleep, clock=lambda: clock[0]))
    assert not res["drained"] and res["reason"] == "inflight_unknown"


def test_ports_and_scrub():
    p = free_tcp_port()
    assert not in_nodeport_range(p)
    b = free_tcp_port_block(4)
    assert not any(in_nodeport_range(x) for x in range(b, b + 4))
    s = scrub("Authorization: Bearer abcdefghijklmnop https://u:pw123@h/x?api_key=SECRET1 sk-abcdefghijklmnopqrs")
    assert "abcdefghijklmnop" not in s and "pw123" not in s and "SECRET1" not in s and "sk-abcdefghijkl" not in s


def test_disagg_preflight():
    preflight(mode="mixed", advertise_host="0.0.0.0", kv_endpoint=None)
    preflight(mode="decode", advertise_host="127.0.0.1", kv_endpoint="ipc:///tmp/pool", single_node=True,
              prefill_gpus=[0, 1], decode_gpus=[2, 3], can_access=lambda a, b: True)
    with pytest.raises(DisaggPreflightError):
        preflight(mode="prefill", advertise_host="0.0.0.0", kv_endpoint=None, single_node=False)
    with pytest.raises(DisaggPreflightError):
        preflight(mode="decode", advertise_host="10.0.0.1", kv_endpoint="tcp://10.0.0.1:5", single_node=False)
    with pytest.raises(DisaggPreflightError):
        preflight(mode="decode", advertise_host="h", kv_endpoint="ipc:///x", prefill_gpus=[0], decode_gpus=[1],
                  can_access=lambda a, b: False)


def _rec(i):
    return WorkerInfo(worker_id=f"w{i}", url=f"http://10.0.0.{i}:9000", model_name="m", kv_block_size=16).to_payload()


def test_k8s_discovery_lifecycle():
    async def go():
        api = FakeK8sClient()
        api.create_pod("ns", "p0", {"app": "w"}, {WORKER_INFO_ANNOTATION: json.dumps(_rec(0))})
        api.create_pod("ns", "other", {"app": "x"}, {WORKER_INFO_ANNOTATION: json.dumps(_rec(9))})
        api.create_pod("ns", "p1", {"app": "w"})  # not yet registered
        reg = KubernetesRegistry(api, "app=w", "ns", reconnect_s=0.01)
        added, removed = [], []
        reg.on_worker_added(lambda w: added.append(w.worker_id))
        reg.on_worker_removed(lambda w: removed.append(w.worker_id))
        await reg.start()
        assert [w.worker_id for w in reg.pool.all()] == ["w0"]
        # the worker on p1 registers itself through its own annotation
        r = K8sRegistration(api, _rec(1), pod_name="p1", namespace="ns", refresh_s=0.01)
        await r.register()
        await asyncio.sleep(0.05)
        assert reg.pool.get("w1") is not None
        # terminating pod: kept but draining (not routed)
        api.mark_terminating("ns", "p0")
        await asyncio.sleep(0.05)
        assert reg.pool.get("w0").status == WorkerStatus.DRAINING
        assert [w.worker_id for w in reg.pool.list_active()] == ["w1"]
        # a delete the watch missed is reconciled by the re-list after a break
        api.delete_pod("ns", "p0", silent=True)
        api.break_watches()
        await asyncio.sleep(0.1)
        assert reg.pool.get("w0") is None and "w0" in removed
        # deregister removes the annotation -> worker removed
        await r.deregister()
        await asyncio.sleep(0.05)
        assert reg.pool.get("w1") is None
        await reg.stop()
        return added

    added = asyncio.run(go())
    assert added == ["w0", "w1"]
    assert merge_patch({"a": {"b": 1, "c": 2}}, {"a": {"b": None, "d": 3}}) == {"a": {"c": 2, "d": 3}}


def _worker(i):
    return WorkerInfo(worker_id=f"w{i}", url="bus://", model_name="m")


def test_bus_transport_stream_admission_cancel():
    async def go():
        bus = InProcessBus()
        started = asyncio.Event()
        cancelled = []

        async def handler(path, body, headers):
            if body.get("hang"):
                started.set()
                try:
                    await asyncio.sleep(60)
                except asyncio.CancelledError:
                    cancelled.append(True)
                    raise
            for i in range(3):
                yield DATA, 200, f"data: {i}\n\n".encode()
            yield DONE, 200, b""

        srv = BusRequestServer(bus, BusRequestClient.token(_worker(0)), handler, max_pending=1)
        await srv.start()
        cl = BusRequestClient(bus, idle_timeout=0.2)
        got = [x async for x in cl.stream(_worker(0), "/v1/completions", {"stream": True})]
        assert [k for k, _, _ in got] == [DATA, DATA, DATA, DONE]
        # idle timeout -> 504 and the worker's task is cancelled
        got = [x async for x in cl.stream(_worker(0), "/v1/completions", {"hang": True})]
        assert got[-1][:2] == (ERROR, 504)
        await asyncio.sleep(0.05)
        assert cancelled and cl.stats["cancels_sent"] == 3
        # admission: a worker at its limit answers 429 without queueing
        srv.max_pending = 0
        got = [x async for x in cl.stream(_worker(0), "/v1/completions", {})]
        assert got == [(ERROR, 429, b"worker at its admission limit")]
        # no such worker: admission times out -> 429
        cl.admit_timeout = 0.05
        got = [x async for x in cl.stream(_worker(5), "/v1/completions", {})]
        assert got[0][1] == 429
        await srv.stop()

    asyncio.run(go())


def test_bus_drain_hands_back_streams():
    async def go():
        bus = InProcessBus()

        async def handler(path, body, headers):
            for i in range(1000):
                yield DATA, 200, b"data: x\n\n"
                await asyncio.sleep(0.01)
            yield DONE, 200, b""

        srv = BusRequestServer(bus, "w0", handler)
        await srv.start()
        cl = BusRequestClient(bus, idle_timeout=5)
        frames = []

        async def consume():
            async for f in cl.stream(_worker(0), "/v1/completions", {"stream": True}):
                frames.append(f)

        t = asyncio.create_task(consume())
        await asyncio.sleep(0.1)
        assert srv.inflight == 1
        ok = await srv.drain(timeout=5, handback_after=0.1)
        await asyncio.wait_for(t, 2)
        # new requests are refused while draining
        srv.max_pending = 10
        refused = [x async for x in cl.stream(_worker(0), "/v1/completions", {})]
        await srv.stop()
        return ok, frames, refused, srv.stats

    ok, frames, refused, stats = asyncio.run(go())
    assert ok and stats["handed_back"] == 1
    assert frames[-1][0] == ERROR and frames[-1][2] == DRAINING_NOTICE.encode()
    assert refused[0][1] == 429


def test_nats_wire_client_against_a_protocol_broker():
    """The NATS protocol client: pub/sub with headers and reply subjects,
    wildcard subscriptions, request/reply, no-responders, and the bus
    request transport (streamed frames, admission, cancel) over it."""
    from infera_b200.common.nats_wire import NatsBus, parse_headers
    from tests.nats_stub import Broker, matches

    assert matches("a.*.c", "a.b.c") and matches("a.>", "a.b.c") and not matches("a.*", "a.b.c")
    assert parse_headers(b"NATS/1.0 503\r\n\r\n") == {"status": "503"}

    async def go():
        br = await Broker().start()
        url = f"nats://127.0.0.1:{br.port}"
        a, b = await NatsBus(url).connect(), await NatsBus(url).connect()
        got = []

        async def on(m):
            got.append(m)

        unsub = await b.subscribe("infera.kv.events.*", on)
        await asyncio.sleep(0.02)
        await a.publish("infera.kv.events.w1", b"\x00\x01payload", headers={"rs-type": "data", "rs-status": "200"},
                        reply="r.1")
        await a.publish("infera.kv.events.w2", b"plain")
        await a.publish("other.subject", b"x")
        for _ in range(100):
            if len(got) >= 2:
                break
            await asyncio.sleep(0.01)
        assert [m.data for m in got] == [b"\x00\x01payload", b"plain"]
        assert got[0].headers == {"rs-type": "data", "rs-status": "200"} and got[0].reply == "r.1"
        unsub()

        async def echo(m):
            await b.publish(m.reply, m.data[::-1])

        await b.subscribe("svc.echo", echo)
        await asyncio.sleep(0.02)
        rs = await asyncio.gather(*[a.request("svc.echo", f"req{i}".encode(), timeout=2.0) for i in range(5)])
        assert [m.data for m in rs] == [f"req{i}".encode()[::-1] for i in range(5)]
        nr = await a.request("svc.nobody", b"", timeout=2.0)   # answered by the broker: no responders
        assert nr.headers.get("status") == "503" and nr.data == b""

        # the bus request transport over NATS
        async def handler(path, body, headers):
            for i in range(3):
                yield DATA, 200, f"data: {i}\n\n".encode()
            yield DONE, 200, b""

        srv = BusRequestServer(b, BusRequestClient.token(_worker(0)), handler)
        await srv.start()
        await asyncio.sleep(0.02)
        cl = BusRequestClient(a, idle_timeout=2.0)
        frames = [x async for x in cl.stream(_worker(0), "/v1/completions", {"stream": True})]
        assert [k for k, _, _ in frames] == [DATA, DATA, DATA, DONE]
        assert frames[0][2] == b"data: 0\n\n"
        cl.admit_timeout = 0.5
        frames = [x async for x in cl.stream(_worker(7), "/v1/completions", {})]   # nobody serves worker 7
        assert frames[0][1] == 429
        await srv.stop()
        await a.close()
        await b.close()
        await br.stop()

    asyncio.run(go())


def test_router_reaches_a_bus_worker_over_nats():
    """Router side: RoutingTransport sends a worker registered with
    request_transport=bus over NATS; worker side: BusRequestServer relays to
    the worker's own HTTP server (here an httpx mock of it)."""
    import httpx

    from infera_b200.common.nats_wire import NatsBus
    from infera_b200.common.request_transport import local_http_handler
    from infera_b200.router.transport import RoutingTransport
    from tests.nats_stub import Broker

    sse = b'data: {"choices":[{"text":"a"}]}\n\ndata: {"choices":[{"text":"b"}]}\n\ndata: [DONE]\n\n'

    def app(req: httpx.Request) -> httpx.Response:
        assert req.url.path == "/v1/completions"
        return httpx.Response(200, content=sse, headers={"content-type": "text/event-stream"})

    async def go():
        br = await Broker().start()
        url = f"nats://127.0.0.1:{br.port}"
        wbus, rbus = await NatsBus(url).connect(), await NatsBus(url).connect()
        w = _worker(3)
        w.request_transport = "bus"
        handler = local_http_handler("http://worker.local", client=httpx.AsyncClient(transport=httpx.MockTransport(app)))
        srv = BusRequestServer(wbus, BusRequestClient.token(w), handler)
        await srv.start()
        await asyncio.sleep(0.02)
        rt = RoutingTransport(bus_client=BusRequestClient(rbus, idle_timeout=2.0))
        frames = [x async for x in rt.stream(w, "/v1/completions", {"stream": True, "prompt": "x"})]
        assert [k for k, _, _ in frames] == [DATA, DATA, DATA, DONE]
        assert frames[-2][2] == b"data: [DONE]\n\n" and srv.stats["served"] == 1
        await srv.stop()
        await wbus.close()
        await rbus.close()
        await br.stop()

    asyncio.run(go())


def test_kv_events_relayed_over_nats():
    """Engine KV events: ZMQ publisher -> worker relay -> NATS
    infera.kv.events.<worker token> -> the router's KV client, which then
    holds the worker's prefix blocks."""
    from infera_b200.common.nats_wire import NatsBus
    from infera_b200.engine.kv_events import KvEventPublisher
    from infera_b200.kv.nats_relay import KvEventNatsRelay
    from infera_b200.router.kv_event.client import KvEventClient
    from tests.nats_stub import Broker

    async def go():
        br = await Broker().start()
        url = f"nats://127.0.0.1:{br.port}"
        wbus, rbus = await NatsBus(url).connect(), await NatsBus(url).connect()
        port = free_tcp_port()
        pub = KvEventPublisher(f"tcp://127.0.0.1:{port}")
        w = WorkerInfo(worker_id="10.0.0.5:9000", url="http://10.0.0.5:9000", model_name="m", kv_block_size=4)
        kv = KvEventClient(use_zmq=False)
        kv.on_worker_added(w)
        await kv.attach_nats(rbus)
        relay = KvEventNatsRelay(wbus, w.worker_id, f"tcp://127.0.0.1:{port}")
        relay.start()
        await asyncio.sleep(0.3)   # ZMQ slow joiner
        pub("BlockStored", {"block_hashes": [11, 12], "parent_block_hash": None,
                            "token_ids": list(range(8)), "block_size": 4})
        pub.flush()
        for _ in range(200):
            if len(kv.cache_view(w.worker_id)) >= 2:
                break
            await asyncio.sleep(0.01)
        assert len(kv.cache_view(w.worker_id)) == 2 and relay.relayed >= 1
        pub("BlockRemoved", {"block_hashes": [12]})
        pub.flush()
        for _ in range(200):
            if len(kv.cache_view(w.worker_id)) == 1:
                break
            await asyncio.sleep(0.01)
        assert len(kv.cache_view(w.worker_id)) == 1
        await relay.stop()
        pub.close()
        await kv.aclose()
        await wbus.close()
        await rbus.close()
        await br.stop()

    asyncio.run(go())

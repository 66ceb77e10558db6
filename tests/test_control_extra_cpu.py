"""Control-plane pieces without their own tests so far: the scaling API
validator, retention -> engine priority, server flags (flag > env >
default), fd passing over a Unix socket, kvd statctl, GPU arch gate."""

import asyncio
import os
import socket

import pytest

from infera_b200.common.worker_pool import EngineType
from infera_b200.router.cache_control import CacheHints, Retention
from infera_b200.router.engine_priority import inject_engine_priority
from infera_b200.server.scaling import DeploymentScaler, ScaleError


class _FakeApi:
    def __init__(self, services):
        self.cr = {"spec": {"services": services}}
        self.patches = []

    async def get_cr(self, group, version, ns, plural, name):
        return self.cr

    async def patch_cr(self, group, version, ns, plural, name, patch):
        self.patches.append(patch)
        for k, v in patch["spec"]["services"].items():
            self.cr["spec"]["services"][k].update(v)


def test_scaler_validates_and_patches():
    api = _FakeApi({"router": {"componentType": "server", "replicas": 1},
                    "prefill": {"componentType": "worker", "role": "prefill", "replicas": 1},
                    "decode": {"componentType": "worker", "role": "decode", "replicas": 2}})
    sc = DeploymentScaler(api, "d1")

    async def go():
        got = await sc.get()
        assert got["services"]["decode"]["replicas"] == 2
        res = await sc.scale({"services": {"prefill": 3, "decode": {"replicas": 4}}})
        assert res["scaled"] == {"prefill": 3, "decode": 4} and api.cr["spec"]["services"]["prefill"]["replicas"] == 3
        for bad, status in (({"services": {"nope": 1}}, 404), ({"services": {"prefill": -1}}, 400),
                            ({"services": {"prefill": True}}, 400), ({}, 400),
                            ({"services": {"prefill": 0, "decode": 0}}, 400)):
            with pytest.raises(ScaleError) as e:
                await sc.scale(bad)
            assert e.value.status == status, bad
        assert len(api.patches) == 1

    asyncio.run(go())


def test_retention_reaches_the_engine():
    hints = CacheHints(retention=Retention.LONG, session_id=None, explicit_hint_seen=True)
    out = inject_engine_priority({"prompt": "x"}, hints, EngineType.INFERA_B200)
    assert out["kv_transfer_params"]["infera_retention"] == "long"
    out = inject_engine_priority({"prompt": "x", "kv_transfer_params": {"room": 3}}, hints, EngineType.INFERA_B200)
    assert out["kv_transfer_params"] == {"room": 3, "infera_retention": "long"}
    out = inject_engine_priority({"prompt": "x"}, hints, "sglang")
    assert out["priority"] == 100 and out["infera_retention"] == "long"
    body = {"prompt": "x"}
    assert inject_engine_priority(body, None, "vllm") is body


def test_server_flags_env_and_defaults(monkeypatch):
    from infera_b200.server.args import parse_server_args

    monkeypatch.setenv("INFERA_REQUEST_MAX_RETRIES", "4")
    monkeypatch.setenv("INFERA_REQUEST_TRANSPORT", "nats")
    a = parse_server_args(["--discovery-backend", "inprocess"])
    assert a.request_max_retries == 4 and a.request_transport == "nats" and a.kv_event_transport == "zmq"
    a = parse_server_args(["--discovery-backend", "inprocess", "--request-max-retries", "2",
                           "--request-transport", "http", "--kv-event-transport", "nats"])
    assert a.request_max_retries == 2 and a.request_transport == "http" and a.kv_event_transport == "nats"
    with pytest.raises(SystemExit):
        parse_server_args(["--discovery-backend", "etcd"])          # etcd needs an endpoint


def test_fd_passing_over_unix_socket(tmp_path):
    from infera_b200.kvd.fd_passing import recv_fd, send_fd

    a, b = socket.socketpair(socket.AF_UNIX, socket.SOCK_STREAM)
    path = tmp_path / "f.bin"
    path.write_bytes(b"shared-bytes")
    fd = os.open(path, os.O_RDONLY)
    send_fd(a, fd)
    got = recv_fd(b)
    assert got != fd and os.pread(got, 12, 0) == b"shared-bytes"
    for x in (fd, got):
        os.close(x)
    a.close()
    b.close()


def test_statctl_reports_daemon_counters(tmp_path, capsys):
    from infera_b200.kvd import statctl
    from infera_b200.kvd.client import KvdClient
    from infera_b200.kvd.server import KvdServer
    from infera_b200.kvd.store import HostStore

    path = str(tmp_path / "kvd.sock")

    async def go():
        srv = KvdServer(path, HostStore(1 << 20))
        await srv.start()
        c = KvdClient(path)
        await c.connect()
        await c.set(b"k" * 8, b"v", "long")
        await c.get(b"k" * 8)
        await c.get(b"m" * 8)
        await c.close()
        d = await statctl.fetch(path)
        await srv.stop()
        return d

    d = asyncio.run(go())
    assert d["entries"] == 1 and d["hits_total"] >= 1 and d["misses_total"] >= 1
    assert 0 < d["hit_rate"] < 1


def test_arch_gate():
    from infera_b200.common.arch import is_supported

    assert is_supported("sm_100a") or is_supported("sm_100")
    assert not is_supported(None) and not is_supported("sm_80")


def test_worker_record_advertises_its_request_transport():
    from infera_b200.engine.worker import build_payload, parse_args
    from infera_b200.utils.tokenizer import load_tokenizer

    tok = load_tokenizer(None, vocab_size=1024)
    a = parse_args(["--model", "tiny-dense", "--port", "9100", "--host", "127.0.0.1"])
    assert build_payload(a, tok)["request_transport"] == "http"
    a = parse_args(["--model", "tiny-dense", "--port", "9100", "--host", "127.0.0.1", "--nats-url",
                    "nats://127.0.0.1:4222", "--disagg-mode", "decode", "--kv-push-endpoint", "tcp://127.0.0.1:7000"])
    d = build_payload(a, tok)
    assert d["request_transport"] == "bus" and d["worker_id"] == "127.0.0.1:9100"
    assert d["disagg_mode"] == "decode" and d["disagg_meta"]["params"]["kv_endpoint"] == "tcp://127.0.0.1:7000"

"""The C++ router (``infera_b200/lib/ib200_router``) against mock workers:
bit-exact block hashing, KV-aware routing from ZMQ events and drain over
etcd, failover, PD body shaping, and the HTTP routes. Mirrors the
reference's Rust router tests (mock upstream workers plus the real app,
``rust/router/tests/functional.rs:35-50``; ZMQ event replay,
``rust/router/tests/kv_event_zmq.rs``)."""

import asyncio
import json
import os
import subprocess
import time

import httpx
import pytest
from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse

from infera_b200.bench.fleet import MockWorker, ServerThread, free_port, run_fleet
from infera_b200.common.etcd_fake import build_app as etcd_app
from infera_b200.server.launch_native import native_argv, router_binary
from infera_b200.utils.hashing import chain_hashes


# release build, plus AddressSanitizer + UndefinedBehaviorSanitizer and
# ThreadSanitizer builds of the same sources: every router started by a test
# logs stderr to a file that must hold no sanitizer report
_SAN_ENV = {"ASAN_OPTIONS": "detect_leaks=0:abort_on_error=0", "UBSAN_OPTIONS": "print_stacktrace=1",
            "TSAN_OPTIONS": "halt_on_error=0:second_deadlock_stack=1"}
_SAN_MARKS = ("ERROR: AddressSanitizer", "runtime error:", "WARNING: ThreadSanitizer", "ERROR: ThreadSanitizer")


@pytest.fixture(scope="module", params=["release", "asan", "tsan"])
def binary(request):
    if request.param == "release":
        return router_binary()
    from infera_b200.build import build_router

    return str(build_router(request.param))


def _start_router(binary, *args):
    import tempfile

    port = free_port()
    log = tempfile.NamedTemporaryFile(prefix="ib200_router_", suffix=".log", delete=False)
    p = subprocess.Popen([binary, "--port", str(port), "--host", "127.0.0.1", *args], stdout=subprocess.DEVNULL,
                         stderr=log, start_new_session=True, env=dict(os.environ, **_SAN_ENV))
    p._log_path = log.name
    url = f"http://127.0.0.1:{port}"
    t0 = time.time()
    while time.time() - t0 < 10:
        try:
            if httpx.get(url + "/health", timeout=1).status_code == 200:
                return p, url
        except httpx.HTTPError:
            time.sleep(0.05)
    p.kill()
    raise RuntimeError("native router did not start")


def _stop(p):
    p.terminate()
    try:
        p.wait(timeout=20)
    except subprocess.TimeoutExpired:
        p.kill()
    path = getattr(p, "_log_path", None)
    if path:
        with open(path, errors="replace") as f:
            text = f.read()
        os.unlink(path)
        hits = [m for m in _SAN_MARKS if m in text]
        assert not hits, text[-6000:]


@pytest.mark.parametrize("bs", [4, 16, 32, 64])
def test_chain_hashes_bit_exact(binary, bs):
    ids = [(i * 7919 + 13) % 128256 for i in range(bs * 9 + 3)]
    r = subprocess.run([binary, "--print-chain-hashes", str(bs)], input=" ".join(map(str, ids)).encode(),
                       stdout=subprocess.PIPE, stderr=subprocess.PIPE, timeout=60, check=True,
                       env=dict(os.environ, **_SAN_ENV))
    assert not [m for m in _SAN_MARKS if m in r.stderr.decode(errors="replace")], r.stderr.decode()[-4000:]
    out = r.stdout.decode().split()
    assert [int(x) for x in out] == chain_hashes(ids, bs)


def test_native_fleet_kv_routing_and_drain():
    res = asyncio.run(run_fleet(workers=3, rate=12.0, duration=8.0, drain_at=4.0, sessions=12, decode_ms=2.0,
                                router_backend="native"))
    assert res["errors"] == 0
    assert res["completed"] >= 40
    assert res["drain"]["drained"] and res["drain"]["router_removed"]
    assert res["prefix_hit_rate"] > 0.5
    assert sum(v > 0 for v in res["router_view_blocks"].values()) >= 2


def _records_file(tmp_path, workers):
    f = tmp_path / "workers.json"
    f.write_text(json.dumps(workers))
    return str(f)


def test_failover_and_routes(binary, tmp_path):
    async def go():
        etcd = ServerThread(etcd_app(), free_port()).start()
        etcd_url = f"http://127.0.0.1:{etcd.port}"
        ws = [MockWorker(i, etcd_url, "m", decode_ms=1.0) for i in range(2)]
        for w in ws:
            await w.start()
        p, url = _start_router(binary, "--etcd-endpoint", etcd_url, "--request-max-retries", "1")
        try:
            t0 = time.time()
            while len(httpx.get(url + "/v1/workers").json()["workers"]) < 2 and time.time() - t0 < 10:
                await asyncio.sleep(0.05)
            ws[0].eng.fail_next = 100
            ws[1].eng.fail_next = 0
            body = {"model": "m", "prompt": list(range(64)), "max_tokens": 4, "ignore_eos": True}
            async with httpx.AsyncClient(timeout=20) as c:
                outs = [await c.post(url + "/v1/completions", json=dict(body, stream=(i % 2 == 0))) for i in range(6)]
                models = (await c.get(url + "/v1/models")).json()
                metrics = (await c.get(url + "/metrics")).text
                missing = await c.get(url + "/v1/nope")
                bad = await c.post(url + "/v1/completions", content=b"{not json")
            return outs, models, metrics, missing, bad
        finally:
            _stop(p)
            for w in ws:
                await w.shutdown(drain_timeout=2)
            etcd.stop()

    outs, models, metrics, missing, bad = asyncio.run(go())
    assert all(r.status_code == 200 for r in outs)
    assert all(r.headers.get("x-infera-request-id") for r in outs)
    assert any(b"[DONE]" in r.content for r in outs)
    assert models["data"][0]["id"] == "m"
    assert 'infera_requests_total{router="native",outcome="ok"} 6' in metrics
    assert "infera_router_failovers_total" in metrics
    assert missing.status_code == 404 and bad.status_code == 400


def _pd_app(role: str, seen: list):
    app = FastAPI()

    @app.post("/v1/completions")
    async def completions(request: Request):
        body = await request.json()
        seen.append(body)
        if role == "prefill":
            return JSONResponse({"choices": [{"text": "x", "finish_reason": "length"}]})

        async def gen():
            for _ in range(3):
                yield b'data: {"choices":[{"text":"y","finish_reason":null}]}\n\n'
            yield b"data: [DONE]\n\n"

        return StreamingResponse(gen(), media_type="text/event-stream")

    return app


def test_pd_nvlink_push_shaping(binary, tmp_path):
    pseen, dseen = [], []
    ps = ServerThread(_pd_app("prefill", pseen), free_port()).start()
    ds = ServerThread(_pd_app("decode", dseen), free_port()).start()
    meta = {"protocol": "b200-nvlink-push", "params": {"kv_endpoint": "ipc://decode-pool"}}
    recs = [{"worker_id": "p0", "url": f"http://127.0.0.1:{ps.port}", "model_name": "m", "disagg_mode": "prefill",
             "disagg_meta": meta, "kv_block_size": 16},
            {"worker_id": "d0", "url": f"http://127.0.0.1:{ds.port}", "model_name": "m", "disagg_mode": "decode",
             "disagg_meta": meta, "kv_block_size": 16}]
    p, url = _start_router(binary, "--discovery-backend", "static", "--static-workers", _records_file(tmp_path, recs))
    try:
        r = httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1, 2, 3], "max_tokens": 10,
                                                      "stream": True}, timeout=20)
        direct = httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1], "max_tokens": 2},
                            headers={"x-worker-instance-id": "d0"}, timeout=20)
    finally:
        _stop(p)
        ps.stop()
        ds.stop()
    assert r.status_code == 200 and r.content.count(b'"y"') == 3 and b"[DONE]" in r.content
    pb, db = pseen[0], dseen[0]
    assert pb["max_tokens"] == 1 and pb["stream"] is False
    assert pb["kv_transfer_params"]["do_remote_decode"] is True
    assert pb["kv_transfer_params"]["decode_kv_endpoint"] == "ipc://decode-pool"
    assert db["max_tokens"] == 10 and db["stream"] is True
    assert db["kv_transfer_params"]["room"] == pb["kv_transfer_params"]["room"]
    assert db["kv_transfer_params"]["infera_retention"] == "long"
    # auto mode ignores gateway headers: that request was routed as a PD pair too
    assert direct.status_code == 200 and len(pseen) == 2


def test_launcher_strips_python_only_flags():
    argv = ["--router-backend", "native", "--enable-profiling", "--kvd-socket-path", "/tmp/x", "--port", "9"]
    assert native_argv(argv) == ["--router-backend", "native", "--port", "9"]
    # the native router enforces the bus requests' overall limit itself
    assert native_argv(["--nats-max-duration", "30"]) == ["--nats-max-duration", "30"]
    assert os.path.exists(router_binary())


def test_native_router_bus_transport_over_nats(binary, tmp_path):
    """--request-transport nats: a worker registered with
    request_transport=bus is reached over NATS (admission, streamed frames,
    unary reply, refusal at the admission limit); two client requests that
    share one X-Infera-Request-Id are both served (each bus attempt has its
    own id); a lost NATS connection answers 503."""
    import asyncio
    import threading

    from infera_b200.common.nats_wire import NatsBus
    from infera_b200.common.request_transport import BusRequestClient, BusRequestServer
    from infera_b200.common.worker_pool import WorkerInfo
    from infera_b200.router.transport import DATA, DONE
    from tests.nats_stub import Broker

    seen = []

    async def handler(path, body, headers):
        seen.append((path, body))
        if body.get("stream"):
            for i in range(3):
                if body.get("max_tokens") == 7:           # slow: overlaps a twin request
                    await asyncio.sleep(0.3)
                yield DATA, 200, f'data: {{"choices":[{{"text":"t{i}"}}]}}\n\n'.encode()
            yield DATA, 200, b"data: [DONE]\n\n"
        else:
            yield DATA, 200, b'{"choices":[{"text":"whole"}]}'
        yield DONE, 200, b""

    loop = asyncio.new_event_loop()
    state = {}
    ready = threading.Event()

    async def serve():
        br = await Broker().start()
        bus = await NatsBus(f"nats://127.0.0.1:{br.port}").connect()
        w = WorkerInfo(worker_id="10.1.2.3:9000", url="bus://", model_name="m")
        srv = BusRequestServer(bus, BusRequestClient.token(w), handler, max_pending=4)
        await srv.start()
        state.update(br=br, bus=bus, srv=srv)
        ready.set()

    th = threading.Thread(target=lambda: (loop.run_until_complete(serve()), loop.run_forever()), daemon=True)
    th.start()
    assert ready.wait(10)
    recs = [{"worker_id": "10.1.2.3:9000", "url": "http://127.0.0.1:1", "model_name": "m", "kv_block_size": 16,
             "request_transport": "bus"}]
    p, url = _start_router(binary, "--discovery-backend", "static", "--static-workers", _records_file(tmp_path, recs),
                           "--request-transport", "nats", "--nats-url", f"nats://127.0.0.1:{state['br'].port}")
    try:
        r = httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1, 2, 3], "max_tokens": 3,
                                                      "stream": True}, timeout=20)
        assert r.status_code == 200 and r.content.count(b'"text":"t') == 3 and b"[DONE]" in r.content
        r = httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1], "max_tokens": 2}, timeout=20)
        assert r.status_code == 200 and r.json()["choices"][0]["text"] == "whole"
        state["srv"].max_pending = 0                      # at its limit: refused without queueing
        r = httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1], "max_tokens": 2}, timeout=20)
        assert r.status_code == 429
        state["srv"].max_pending = 4
        import concurrent.futures

        def twin():
            return httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1], "max_tokens": 7,
                                                             "stream": True},
                              headers={"X-Infera-Request-Id": "same-id"}, timeout=20)

        with concurrent.futures.ThreadPoolExecutor(2) as ex:
            rs = list(ex.map(lambda _: twin(), range(2)))
        for r in rs:
            assert r.status_code == 200 and r.content.count(b'"text":"t') == 3, r.content
            assert r.headers.get("x-infera-request-id") == "same-id"
        loop.call_soon_threadsafe(state["br"].kick)       # the broker goes away
        time.sleep(0.5)
        r = httpx.post(url + "/v1/completions", json={"model": "m", "prompt": [1], "max_tokens": 2}, timeout=20)
        assert r.status_code == 503 and "NATS connection lost" in r.text
    finally:
        _stop(p)

        async def down():
            await state["srv"].stop()
            await state["bus"].close()
            await state["br"].stop()

        asyncio.run_coroutine_threadsafe(down(), loop).result(10)
        loop.call_soon_threadsafe(loop.stop)
    assert [s[0] for s in seen] == ["/v1/completions"] * 4
    assert seen[0][1]["max_tokens"] == 3 and seen[0][1]["stream"] is True


def _train_bpe(path, family: str):
    """A small byte-level BPE tokenizer.json of the given family, trained
    with the `tokenizers` library on a multilingual random corpus."""
    import random

    from tokenizers import Regex, Tokenizer, models, normalizers, pre_tokenizers, trainers

    split = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"
             r"|\s*[\r\n]+|\s+(?!\S)|\s+")
    rng = random.Random(0)
    words = ["hello", "world", "don't", "I'm", "THEY'RE", "naïve", "café", "日本語", "한국어", "Привет", "αβγ", "123456",
             "3.14", "x=y+1;", "<tag>", "  ", "\t", "\n\n", "foo_bar", "!!!", "—", "😀", "٣٤٥"]
    corpus = [" ".join(rng.choice(words) for _ in range(30)) for _ in range(1500)]
    if family == "gpt2":
        t = Tokenizer(models.BPE())
        t.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=True, use_regex=True)
    else:
        t = Tokenizer(models.BPE(ignore_merges=family == "llama3"))
        if family == "qwen2":
            split = split.replace(r"\p{N}{1,3}", r"\p{N}")
            t.normalizer = normalizers.NFC()
        t.pre_tokenizer = pre_tokenizers.Sequence([pre_tokenizers.Split(Regex(split), "isolated"),
                                                   pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    t.train_from_iterator(corpus, trainers.BpeTrainer(vocab_size=1200, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                                      special_tokens=["<|begin_of_text|>", "<|user|>"]))
    t.save(str(path))
    return t


@pytest.mark.parametrize("family", ["llama3", "qwen2", "gpt2"])
def test_bpe_tokenizer_matches_tokenizers_library(binary, tmp_path, family):
    """The router's byte-level BPE (split pattern scanned by hand, merges,
    added tokens, NFC refusal) gives the same ids as the `tokenizers`
    library with add_special_tokens=False, the engine's encoding."""
    import random

    path = tmp_path / f"{family}.json"
    tok = _train_bpe(path, family)
    rng = random.Random(1)
    pieces = ["hello", "World", "don't", "I'M", "we'LL", "'S", "naïve", "café", "über", "日本語", "中文", "Привет",
              "1", "12", "1234567", "3.14159", "x=y+1;", " ", "  ", "\t", "\n", "\n\n", " \n ", "\r\n", "é", "!!!",
              "...", "😀", "٣٤٥", "<|begin_of_text|>", "<|user|>", " ", "　", "Ⅻ", "½", "'", "'x"]
    texts = ["".join(rng.choice(pieces) + rng.choice(["", " "]) for _ in range(rng.randint(1, 10)))
             for _ in range(600)] + ["", " ", "  a", "a  ", "'s'S'Re", "   \n\n  x", "x\n  \ny"]
    r = subprocess.run([binary, "--tokenize", str(path)], input=("\n".join(json.dumps(t) for t in texts) + "\n").encode(),
                       capture_output=True, timeout=120, env=dict(os.environ, **_SAN_ENV))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    assert not [m for m in _SAN_MARKS if m in r.stderr.decode(errors="replace")], r.stderr.decode()[-4000:]
    outs = r.stdout.decode().splitlines()
    assert len(outs) == len(texts)
    refused = 0
    for t, o in zip(texts, outs):
        got = json.loads(o)
        if got is None:
            refused += 1
            assert family == "qwen2" and "́" in t        # only texts NFC would change are refused
            continue
        assert got == tok.encode(t, add_special_tokens=False).ids, repr(t)
    assert refused < len(texts) // 2


def _self_signed(tmp_path):
    """A CA-less self-signed certificate for 127.0.0.1 (it is its own CA bundle)."""
    import datetime
    import ipaddress

    from cryptography import x509
    from cryptography.hazmat.primitives import hashes, serialization
    from cryptography.hazmat.primitives.asymmetric import ec
    from cryptography.x509.oid import NameOID

    key = ec.generate_private_key(ec.SECP256R1())
    name = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, "fake-apiserver")])
    now = datetime.datetime.now(datetime.timezone.utc)
    cert = (x509.CertificateBuilder().subject_name(name).issuer_name(name).public_key(key.public_key())
            .serial_number(x509.random_serial_number()).not_valid_before(now - datetime.timedelta(minutes=5))
            .not_valid_after(now + datetime.timedelta(days=1))
            .add_extension(x509.SubjectAlternativeName([x509.IPAddress(ipaddress.ip_address("127.0.0.1"))]),
                           critical=False)
            .add_extension(x509.BasicConstraints(ca=True, path_length=None), critical=True)
            .sign(key, hashes.SHA256()))
    cf, kf = tmp_path / "apiserver.crt", tmp_path / "apiserver.key"
    cf.write_bytes(cert.public_bytes(serialization.Encoding.PEM))
    kf.write_bytes(key.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.TraditionalOpenSSL,
                                     serialization.NoEncryption()))
    return str(cf), str(kf)


@pytest.mark.parametrize("tls", [False, True])
def test_kubernetes_discovery(binary, tmp_path, tls):
    """Pods with the worker-info annotation become workers (list, then the
    watch), a deletionTimestamp makes one draining (listed, not routed), a
    DELETED event removes it, and a delete the watch missed is reconciled by
    the re-list after the watch breaks. TLS: the API server's certificate is
    verified against the given CA bundle and the bearer token is sent."""
    from infera_b200.common.k8s_client import FakeK8sClient
    from infera_b200.common.k8s_fake_server import build_app as k8s_app

    fake = FakeK8sClient()
    token = tmp_path / "token"
    token.write_text("s3cret\n")
    cert = _self_signed(tmp_path) if tls else (None, None)
    srv = ServerThread(k8s_app(fake, require_token="s3cret"), free_port(), ssl_certfile=cert[0],
                       ssl_keyfile=cert[1]).start()
    labels = {"app": "infera-worker"}

    def rec(i):
        return json.dumps({"worker_id": f"w{i}", "url": f"http://127.0.0.1:{40000 + i}", "model_name": "m"})

    def on_loop(fn, *a):
        # mutate the fake on the server's event loop (its watch queues live there)
        import threading

        done = threading.Event()

        def run():
            fn(*a)
            done.set()

        srv.server_loop.call_soon_threadsafe(run)
        assert done.wait(5)

    for i in range(2):
        fake.create_pod("infera", f"pod{i}", labels, {"infera.amd.com/worker-info": rec(i)})
    fake.create_pod("infera", "other", {"app": "else"}, {"infera.amd.com/worker-info": rec(9)})
    scheme = "https" if tls else "http"
    args = ["--discovery-backend", "kubernetes", "--k8s-label-selector", "app=infera-worker", "--k8s-namespace",
            "infera", "--k8s-api-url", f"{scheme}://127.0.0.1:{srv.port}", "--k8s-token-file", str(token)]
    if tls:
        args += ["--k8s-ca-file", cert[0]]
    p, url = _start_router(binary, *args)

    def workers():
        return {w["worker_id"]: w.get("status") for w in httpx.get(url + "/v1/workers").json()["workers"]}

    def wait_for(pred, what):
        t0 = time.time()
        while time.time() - t0 < 10:
            if pred(workers()):
                return
            time.sleep(0.05)
        raise AssertionError(f"{what}: {workers()}")

    try:
        wait_for(lambda w: set(w) == {"w0", "w1"}, "listed pods")
        on_loop(fake.create_pod, "infera", "pod2", labels, {"infera.amd.com/worker-info": rec(2)})
        wait_for(lambda w: "w2" in w, "watched ADDED")
        on_loop(fake.mark_terminating, "infera", "pod1")
        wait_for(lambda w: w.get("w1") == "draining", "terminating pod draining")
        assert httpx.get(url + "/health").json()["workers"] == 2
        on_loop(fake.delete_pod, "infera", "pod1")
        wait_for(lambda w: "w1" not in w, "DELETED")
        on_loop(fake.delete_pod, "infera", "pod0", True)       # the watch misses it
        on_loop(fake.break_watches)
        wait_for(lambda w: set(w) == {"w2"}, "re-list reconciles the missed delete")
    finally:
        _stop(p)
        srv.stop()

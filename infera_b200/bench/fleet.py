"""CPU fleet benchmark for the router plumbing (serving config 1).

Everything runs in one process on localhost, over the real wire paths:
an in-memory etcd v3 JSON gateway; N mock engine workers (each registers
with a 30 s lease and heartbeats, publishes KV events on its own ZMQ PUB
socket); the router (KV-aware policy, etcd discovery, ZMQ event client)
behind the FastAPI front door; and the open-loop trace replayed by the HTTP
load generator against the router. Optionally one worker receives the
shutdown sequence mid-run (heartbeat stop -> deregister -> drain -> stop)
and the run reports whether any request failed. That worker runs as its
own process (``--serve-worker`` mode of this module) and the shutdown is a
real SIGTERM: its signal handler stops the heartbeat, deregisters, drains
its in-flight requests and exits.

    python -m infera_b200.bench.fleet [--workers 4] [--rate 20] [--duration 60] [--drain-at 30]

Reports the prefix-hit rate seen by the workers, TTFT p50 / p99, request
errors and the per-worker request split.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import socket
import sys
import threading
import time

from infera_b200.bench.slo import percentile


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class ServerThread:
    """A uvicorn server on a background thread."""

    def __init__(self, app, port: int, ssl_certfile: str | None = None, ssl_keyfile: str | None = None):
        import uvicorn

        self.port = port
        self.server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning",
                                                   access_log=False, ssl_certfile=ssl_certfile,
                                                   ssl_keyfile=ssl_keyfile))
        self.server_loop = None
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        import asyncio

        loop = asyncio.new_event_loop()
        asyncio.set_event_loop(loop)
        self.server_loop = loop
        loop.run_until_complete(self.server.serve())

    def start(self) -> "ServerThread":
        self.thread.start()
        t0 = time.time()
        while not self.server.started and time.time() - t0 < 30:
            time.sleep(0.02)
        return self

    def stop(self) -> None:
        self.server.should_exit = True
        self.thread.join(timeout=10)


class MockWorker:
    def __init__(self, idx: int, etcd_url: str, model: str, *, capacity_blocks=4096, prefill_ms=0.05,
                 decode_ms=10.0, vocab=32000, port: int | None = None, engine: str = "infera-b200",
                 word_ids: bool = False):
        from infera_b200.bench.mock_engine import MockEngine, build_mock_app
        from infera_b200.common.worker_pool import EngineType, KvRegistrationMetadata, WorkerInfo
        from infera_b200.engine.kv_events import KvEventPublisher
        from infera_b200.utils.tokenizer import ByteTokenizer, canary

        self.port = port or free_port()
        ev_port = free_port()
        self.ev_endpoint = f"tcp://127.0.0.1:{ev_port}"
        self.pub = KvEventPublisher(self.ev_endpoint, flush_ms=0.0)
        self.eng = MockEngine(capacity_blocks=capacity_blocks, prefill_ms_per_token=prefill_ms,
                              decode_ms_per_token=decode_ms, vocab=vocab, publisher=self.pub, seed=idx)
        self.server = ServerThread(build_mock_app(self.eng, model, word_ids=word_ids), self.port)
        tok = ByteTokenizer(vocab_size=vocab)
        kv = KvRegistrationMetadata(engine_block_size=16, index_block_size=16, tokenizer=tok.name,
                                    tokenizer_digest=tok.digest(), tokenizer_canary=canary(tok),
                                    events_endpoint=self.ev_endpoint)
        self.info = WorkerInfo(worker_id=f"127.0.0.1:{self.port}", url=f"http://127.0.0.1:{self.port}",
                               model_name=model, engine=EngineType(engine), kv_events_endpoint=self.ev_endpoint,
                               kv_block_size=16, kv=kv)
        self.etcd_url = etcd_url
        self.reg = None
        self.hb = None

    @property
    def worker_id(self) -> str:
        return self.info.worker_id

    def requests(self) -> int:
        return self.eng.stats["requests"]

    async def start(self) -> None:
        from infera_b200.common.registration import EtcdRegistration

        self.server.start()
        self.reg = EtcdRegistration(self.etcd_url, self.info.to_payload())
        await self.reg.register()
        self.hb = asyncio.create_task(self.reg.heartbeat_loop())

    async def shutdown(self, drain_timeout: float = 60.0) -> dict:
        """Heartbeat off -> deregister -> drain in-flight -> stop."""
        t0 = time.monotonic()
        if self.hb is not None:
            self.hb.cancel()
        await self.reg.deregister()
        t_dereg = time.monotonic() - t0
        while self.eng.inflight > 0 and time.monotonic() - t0 < drain_timeout:
            await asyncio.sleep(0.01)
        drained = self.eng.inflight == 0
        self.eng.draining = True
        self.server.stop()
        self.pub.close()
        await self.reg.close()
        return {"deregister_s": t_dereg, "drain_s": time.monotonic() - t0, "drained": drained}


class WorkerProcess:
    """A mock worker in its own process (``--serve-worker``), shut down by a
    real SIGTERM."""

    def __init__(self, idx: int, etcd_url: str, model: str, *, decode_ms: float = 10.0, prefill_ms: float = 0.05,
                 engine: str = "infera-b200", word_ids: bool = False):
        self.port = free_port()
        self.cmd = [sys.executable, "-m", "infera_b200.bench.fleet", "--serve-worker", "--etcd", etcd_url,
                    "--index", str(idx), "--model", model, "--port", str(self.port), "--decode-ms", str(decode_ms),
                    "--prefill-ms", str(prefill_ms), "--engine", engine] + (["--word-ids"] if word_ids else [])
        self.proc = None
        self.worker_id = f"127.0.0.1:{self.port}"
        self.final: dict = {}

    def start(self) -> "WorkerProcess":
        import subprocess

        self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                                     start_new_session=True)
        line = self.proc.stdout.readline()          # {"worker_id": ...} once registered
        if not line:
            raise RuntimeError("mock worker process did not start")
        self.worker_id = json.loads(line)["worker_id"]
        return self

    def sigterm(self) -> None:
        import signal

        self.t_term = time.monotonic()
        self.proc.send_signal(signal.SIGTERM)

    async def wait_exit(self, timeout: float = 60.0) -> dict:
        t0 = time.monotonic()
        while self.proc.poll() is None and time.monotonic() - t0 < timeout:
            await asyncio.sleep(0.01)
        rc = self.proc.poll()
        out = self.proc.stdout.read() if rc is not None else ""
        for line in out.splitlines():
            try:
                self.final = json.loads(line)
            except ValueError:
                pass
        return {"exit_code": rc, "sigterm_to_exit_s": time.monotonic() - self.t_term, **self.final}

    def requests(self) -> int:
        return int(self.final.get("requests", 0))

    def kill(self) -> None:
        if self.proc is not None and self.proc.poll() is None:
            self.proc.kill()
            self.proc.wait(timeout=10)


def serve_worker(a) -> None:
    """``--serve-worker``: one mock worker; SIGTERM = heartbeat off ->
    deregister -> drain in-flight -> stop, then a JSON line with the timings
    and the request count, exit 0."""
    import signal

    async def go():
        w = MockWorker(a.index, a.etcd, a.model, decode_ms=a.decode_ms, prefill_ms=a.prefill_ms, port=a.port,
                       engine=a.engine, word_ids=a.word_ids)
        await w.start()
        print(json.dumps({"worker_id": w.info.worker_id}), flush=True)
        stop = asyncio.Event()
        asyncio.get_running_loop().add_signal_handler(signal.SIGTERM, stop.set)
        await stop.wait()
        info = await w.shutdown()
        info["requests"] = w.eng.stats["requests"]
        print(json.dumps(info), flush=True)

    asyncio.run(go())


async def run_fleet(*, workers: int = 4, rate: float = 20.0, duration: float = 60.0, drain_at: float | None = 30.0,
                    sessions: int = 64, policy: str = "kv-aware", seed: int = 0, trace: str = "router-plumbing",
                    decode_ms: float = 10.0, prefill_ms: float = 0.05, router_backend: str = "python",
                    text_prompts: bool = False) -> dict:
    """``text_prompts``: prompts go as ``t<id>`` word text that the router
    tokenizes with a word-level ``tokenizer.json`` (always on for the
    reference router, which accepts text only); else as token ids.
    ``router_backend``: "python" (the router stack in this process),
    "native" (the C++ router binary as a child process) or "reference" (the
    reference's router, ``python -m infera.server``, as a child process)."""
    from types import SimpleNamespace

    from infera_b200.common.etcd_fake import build_app as etcd_app
    from infera_b200.server.__main__ import build_router_stack
    from infera_b200.server.app import build_app

    model = "mock-model"
    text_prompts = text_prompts or router_backend == "reference"
    tok_dir = None
    if text_prompts:
        from infera_b200.bench.hf_model_dir import write_model_dir

        tok_dir = write_model_dir("/tmp/infera_fleet_tokenizer", "llama-3.1-8b")   # word-level t<id> tokenizer
    etcd = ServerThread(etcd_app(), free_port()).start()
    etcd_url = f"http://127.0.0.1:{etcd.port}"
    # the worker that is shut down mid-run is a separate process (SIGTERM)
    n_proc = 1 if drain_at is not None and workers > 1 else 0
    # the mocks speak vLLM's API and KV events; the reference's registry only
    # accepts the engine types it knows
    eng_t = "vllm" if router_backend == "reference" else "infera-b200"
    ws = [MockWorker(i, etcd_url, model, decode_ms=decode_ms, prefill_ms=prefill_ms, engine=eng_t,
                     word_ids=text_prompts) for i in range(workers - n_proc)]
    for w in ws:
        await w.start()
    if n_proc:
        ws.append(WorkerProcess(workers - 1, etcd_url, model, decode_ms=decode_ms, prefill_ms=prefill_ms,
                                engine=eng_t, word_ids=text_prompts).start())
    native = None
    state = None
    if router_backend in ("native", "reference"):
        import os
        import subprocess

        rport = free_port()
        if router_backend == "native":
            from infera_b200.server.launch_native import router_binary

            cmd = [router_binary(), "--port", str(rport), "--host", "127.0.0.1", "--discovery-backend", "etcd",
                   "--etcd-endpoint", etcd_url, "--router-policy", policy, "--log-level", "warning"]
            if tok_dir:
                cmd += ["--router-tokenizer-path", os.path.join(tok_dir, "tokenizer.json")]
            env = None
        else:
            # the reference's own router, unmodified (installed under baseline/_ref)
            ref = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                               "baseline", "_ref")
            env = dict(os.environ, PYTHONPATH=ref, HF_HUB_OFFLINE="1", TRANSFORMERS_OFFLINE="1")
            cmd = [sys.executable, "-m", "infera.server", "--discovery-backend", "etcd", "--etcd-endpoint",
                   etcd_url.replace("http://", ""), "--router-policy", policy, "--host", "127.0.0.1",
                   "--port", str(rport), "--router-tokenizer-path", tok_dir, "--request-transport", "http",
                   "--kv-event-transport", "zmq"]
        log = open(os.path.join(os.environ.get("INFERA_LOG_DIR", "/tmp"), f"fleet_router_{router_backend}.log"), "w")
        native = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, start_new_session=True, env=env)
        router_url = f"http://127.0.0.1:{rport}"
    else:
        args = SimpleNamespace(router_policy=policy, router_tokenizer_path=tok_dir, kv_overlap_weight=1.0,
                               kv_prefill_overlap_weight=None, kv_decode_overlap_weight=None,
                               breaker_failure_threshold=3, breaker_cooldown_s=5.0, breaker_max_cooldown_s=60.0,
                               discovery_backend="etcd", etcd_endpoint=etcd_url, etcd_prefix="/infera/workers/",
                               request_max_retries=1, migration_limit=0, router_mode="auto", enable_profiling=True,
                               enable_scaling_api=False, scaling_deployment=None, kvd_socket_path=None, block_size=16,
                               k8s_label_selector=None, k8s_namespace=None)
        state = build_router_stack(args)
        app = build_app(state)
        app.router.on_startup.append(state.registry.start)
        router = ServerThread(app, free_port()).start()
        router_url = f"http://127.0.0.1:{router.port}"

    import httpx

    async def listed() -> list[str]:
        if state is not None:
            return [w.worker_id for w in state.registry.pool.list_active()]
        try:
            async with httpx.AsyncClient() as c:
                r = await c.get(router_url + "/v1/workers", timeout=2)
            return [w["worker_id"] for w in r.json()["workers"] if w.get("status", "active") == "active"]
        except Exception:
            return []

    async def view_size(wid: str) -> int:
        if state is not None:
            return len(state.policy.kv_client.cache_view(wid))
        async with httpx.AsyncClient() as c:
            r = await c.get(router_url + f"/v1/admin/cache-view/{wid}", timeout=5)
        return int(r.json().get("num_blocks", 0)) if r.status_code == 200 else 0

    try:
        return await _drive(ws, listed, view_size, router_url, workers, drain_at, trace, sessions, rate, duration, seed,
                            model, policy, text_prompts=router_backend == "reference")
    finally:
        if native is not None:
            native.terminate()
            try:
                native.wait(timeout=10)
            except Exception:
                native.kill()
        else:
            router.stop()
        for w in ws:
            if isinstance(w, WorkerProcess):
                w.kill()
            elif w.server.thread.is_alive():
                await w.shutdown(drain_timeout=5)
        if state is not None:
            await state.registry.stop()
        etcd.stop()


async def _drive(ws, listed, view_size, router_url, workers, drain_at, trace, sessions, rate, duration, seed, model,
                 policy, text_prompts: bool = False) -> dict:
    from infera_b200.bench.http_loadgen import run as loadgen

    t_wait = time.time()
    while len(await listed()) < workers and time.time() - t_wait < 90:
        await asyncio.sleep(0.05)
    drain_info = {}

    async def drainer():
        await asyncio.sleep(drain_at)
        t0 = time.monotonic()
        victim = ws[-1]
        victim.sigterm()
        # the router stops listing the victim (it deregistered on SIGTERM)
        while victim.worker_id in await listed() and time.monotonic() - t0 < 5.0:
            await asyncio.sleep(0.005)
        info = {"router_removed": victim.worker_id not in await listed(),
                "sigterm_to_unlisted_s": time.monotonic() - t0}
        info.update(await victim.wait_exit())
        info["t"] = time.monotonic() - t0
        drain_info.update(info)

    dtask = asyncio.create_task(drainer()) if drain_at is not None and workers > 1 else None
    res = await loadgen(router_url, model, trace, list(range(sessions)), rate, duration, seed, stop_after_s=30.0,
                        text_prompts=text_prompts)
    if dtask is not None:
        await dtask
    recs = [r for r in res["records"] if r["token_times"]]
    ttfts = [r["token_times"][0] - r["arrival"] for r in recs]
    prompt = sum(r["prompt_len"] for r in recs)
    cached = sum(r["cached_len"] for r in recs)
    split = {w.worker_id: w.requests() for w in ws}
    view = {wid: await view_size(wid) for wid in split} if policy == "kv-aware" else {}
    out = {
        "requests": len(res["records"]), "completed": len(recs), "errors": res["errors"],
        "prefix_hit_rate": cached / max(1, prompt),
        "ttft_p50_ms": 1000 * percentile(ttfts, 50), "ttft_p99_ms": 1000 * percentile(ttfts, 99),
        "per_worker_requests": split, "router_view_blocks": view, "drain": drain_info,
    }
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workers", type=int, default=4)
    ap.add_argument("--rate", type=float, default=20.0)
    ap.add_argument("--duration", type=float, default=60.0)
    ap.add_argument("--drain-at", type=float, default=30.0)
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--policy", default="kv-aware")
    ap.add_argument("--router-backend", choices=("python", "native", "reference"), default="python",
                    help="reference: the reference's own router (baseline/_ref) in front of the same mock fleet")
    ap.add_argument("--text-prompts", action="store_true",
                    help="send prompts as t<id> word text tokenized by the router (word-level tokenizer.json)")
    ap.add_argument("--serve-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--etcd", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--index", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--model", default="mock-model", help=argparse.SUPPRESS)
    ap.add_argument("--port", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--decode-ms", type=float, default=10.0)
    ap.add_argument("--prefill-ms", type=float, default=0.05)
    ap.add_argument("--engine", default="infera-b200", help=argparse.SUPPRESS)
    ap.add_argument("--word-ids", action="store_true", help=argparse.SUPPRESS)
    a = ap.parse_args(argv)
    if a.serve_worker:
        serve_worker(a)
        return
    res = asyncio.run(run_fleet(workers=a.workers, rate=a.rate, duration=a.duration, drain_at=a.drain_at,
                                sessions=a.sessions, policy=a.policy, router_backend=a.router_backend,
                                text_prompts=a.text_prompts))
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()

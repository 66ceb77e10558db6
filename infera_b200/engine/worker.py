"""``python -m infera_b200.engine.worker``: one engine instance as a fleet
worker.

Lifecycle (``infera/engine/vllm/__main__.py:142-405``, for this framework's
own engine):

1. start the engine core (by default a child process that owns the GPU, the
   KV-event publisher and the step loop, reached over ZMQ IPC; or an
   already-running core given by ``--attach-core``; or, with
   ``--in-process``, a thread of this process) and the worker HTTP app;
2. serve HTTP, then register (etcd lease + heartbeat, or the in-process
   registry) with a record carrying the KV metadata (block size, tokenizer
   digest and canary, events endpoint);
3. on SIGTERM / SIGINT: stop the heartbeat, DEREGISTER FIRST (the router
   stops sending), drain in-flight requests (exact count, bounded by
   ``--drain-timeout``; optionally hand the stragglers back for migration),
   then stop the engine and the server.
"""

from __future__ import annotations

import argparse
import asyncio
import logging
import signal
import socket

logger = logging.getLogger(__name__)


def _connect_addr(bind: str, host: str) -> str:
    """A ZMQ bind address as peers connect to it (a wildcard host becomes
    the advertised one)."""
    for wild in ("tcp://*:", "tcp://0.0.0.0:"):
        if bind.startswith(wild):
            return f"tcp://{host}:" + bind[len(wild):]
    return bind


def worker_id(args) -> str:
    host = args.advertise_host or args.host
    if host in ("0.0.0.0", ""):
        host = socket.gethostname()
    return f"{host}:{args.port}"


def build_payload(args, tokenizer) -> dict:
    from infera_b200.common.worker_pool import (DisaggMode, EngineType, KvRegistrationMetadata, WorkerInfo)
    from infera_b200.utils.tokenizer import canary

    host = args.advertise_host or args.host
    if host in ("0.0.0.0", ""):
        host = socket.gethostname()
    wid = f"{host}:{args.port}"
    meta = {}
    if args.disagg_mode != "mixed":
        meta = {"protocol": "b200-nvlink-push", "params": {"kv_endpoint": args.kv_push_endpoint or ""}}
    idx_ep = getattr(args, "kv_index_endpoint", None)
    tiers = ["device"] + (["host", "disk"] if args.kv_tier else [])
    kv = KvRegistrationMetadata(engine_block_size=args.page_size, index_block_size=args.page_size,
                                tokenizer=tokenizer.name, tokenizer_digest=tokenizer.digest(),
                                tokenizer_canary=canary(tokenizer), supports_events=bool(idx_ep),
                                events_endpoint=_connect_addr(idx_ep, host) if idx_ep else None,
                                snapshot_endpoint=f"http://{host}:{args.port}", tiers=tiers)
    w = WorkerInfo(worker_id=wid, url=f"http://{host}:{args.port}", model_name=args.served_model_name or args.model,
                   engine=EngineType.INFERA_B200, disagg_mode=DisaggMode(args.disagg_mode), disagg_meta=meta,
                   kv_events_endpoint=args.kv_events_endpoint, kv_block_size=args.page_size, kv=kv,
                   dp_rank=args.dp_rank, dp_size=args.dp_size,
                   request_transport="bus" if getattr(args, "nats_url", None) else "http")
    return w.to_payload()


def parse_args(argv=None):
    p = argparse.ArgumentParser(prog="python -m infera_b200.engine.worker")
    p.add_argument("--model", default="llama-3.1-8b")
    p.add_argument("--served-model-name", default=None)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--advertise-host", default=None)
    p.add_argument("--port", type=int, default=9000)
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--tp-size", type=int, default=1,
                   help="tensor-parallel ranks of the engine core (launched with torch.distributed.run)")
    p.add_argument("--first-device", type=int, default=0,
                   help="with --tp-size: rank r runs on cuda:(first + r)")
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--max-num-seqs", type=int, default=128)
    p.add_argument("--max-batched-tokens", type=int, default=2048)
    p.add_argument("--mixed-prefill-tokens", type=int, default=256,
                   help="prompt tokens per step while sequences are decoding (0: no cap)")
    p.add_argument("--gpu-memory-utilization", type=float, default=0.90)
    p.add_argument("--num-pages", type=int, default=None)
    p.add_argument("--no-cuda-graphs", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--etcd-endpoint", default=None)
    p.add_argument("--k8s-register", action="store_true",
                   help="register through this Pod's worker-info annotation (in-cluster service account)")
    p.add_argument("--kv-events-endpoint", default=None, help="ZMQ PUB bind address, e.g. tcp://127.0.0.1:5557")
    p.add_argument("--kv-index-endpoint", default=None,
                   help="ZMQ PUB bind address of the tier-aware KV index events (registered as kv.events_endpoint)")
    p.add_argument("--disagg-mode", choices=("mixed", "prefill", "decode"), default="mixed")
    p.add_argument("--kv-push-endpoint", default=None)
    p.add_argument("--drain-timeout", type=float, default=30.0)
    p.add_argument("--handback-after", type=float, default=None)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--kv-tier", default=None, help="host:<GiB>[:<nvme dir>] or kvd:<socket>")
    p.add_argument("--in-process", action="store_true", help="run the engine on a thread of this process")
    p.add_argument("--attach-core", default=None, help="IN,OUT ipc addresses of a running engine core")
    p.add_argument("--dp-rank", type=int, default=None,
                   help="data-parallel attention rank this worker serves (registered for DP-rank routing)")
    p.add_argument("--dp-size", type=int, default=1)
    p.add_argument("--nats-jetstream", action="store_true",
                   help="with --nats-url: KV events into the INFERA_KV_EVENTS stream and this worker's view into "
                        "the INFERA_KV_VIEWS bucket; requests from the INFERA_REQUESTS work queue")
    p.add_argument("--nats-url", default=None,
                   help="also serve requests over NATS (infera.req.<worker token>); registers request_transport=bus")
    p.add_argument("--log-level", default="info")
    return p.parse_args(argv)


def _core_cmd(args, in_addr: str, out_addr: str) -> list[str]:
    import sys

    launch = [sys.executable, "-m", "infera_b200.engine.core_ipc"]
    tp = getattr(args, "tp_size", 1)
    if tp > 1:
        # one process per GPU: rank 0 serves the core's IPC sockets, the
        # others follow its step commands
        from infera_b200.common.net import free_tcp_port

        launch = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
                  "--master-addr", "127.0.0.1", "--master-port", str(free_tcp_port()), "-m",
                  "infera_b200.engine.core_ipc", "--tp-size", str(tp), "--first-device", str(args.first_device)]
    cmd = launch + ["--in", in_addr, "--out", out_addr,
           "--model", args.model, "--device", args.device, "--page-size", str(args.page_size),
           "--max-num-seqs", str(args.max_num_seqs), "--max-batched-tokens", str(args.max_batched_tokens),
           "--mixed-prefill-tokens", str(args.mixed_prefill_tokens),
           "--gpu-memory-utilization", str(args.gpu_memory_utilization), "--seed", str(args.seed)]
    if args.num_pages:
        cmd += ["--num-pages", str(args.num_pages)]
    if args.no_cuda_graphs:
        cmd.append("--no-cuda-graphs")
    if args.kv_events_endpoint:
        cmd += ["--kv-events-endpoint", args.kv_events_endpoint]
    if getattr(args, "kv_index_endpoint", None):
        cmd += ["--kv-index-endpoint", args.kv_index_endpoint, "--kv-index-publisher", worker_id(args),
                "--kv-index-model", args.served_model_name or args.model,
                "--kv-index-compat", getattr(args, "_compat", "")]
    if args.kv_tier:
        cmd += ["--kv-tier", args.kv_tier]
    cmd += ["--disagg-mode", args.disagg_mode]
    if args.kv_push_endpoint:
        cmd += ["--kv-push-endpoint", args.kv_push_endpoint]
    return cmd


async def start_engine(args):
    """Returns (serving engine, vocab size, shutdown coroutine factory)."""
    if args.in_process:
        from infera_b200.engine.async_engine import AsyncEngine
        from infera_b200.engine.kv_events import KvEventPublisher
        from infera_b200.engine.llm_engine import EngineConfig, LLMEngine

        pub = KvEventPublisher(args.kv_events_endpoint) if args.kv_events_endpoint else None
        ecfg = EngineConfig(model=args.model, page_size=args.page_size, max_num_seqs=args.max_num_seqs,
                            max_batched_tokens=args.max_batched_tokens,
                            mixed_prefill_tokens=args.mixed_prefill_tokens,
                            gpu_memory_utilization=args.gpu_memory_utilization, num_pages=args.num_pages,
                            use_cuda_graphs=not args.no_cuda_graphs, seed=args.seed, kv_tier=args.kv_tier,
                            disagg_mode=args.disagg_mode, kv_push_endpoint=args.kv_push_endpoint)
        eng = LLMEngine(ecfg, device=args.device, event_sink=pub)
        feed = None
        if getattr(args, "kv_index_endpoint", None):
            from infera_b200.engine.kv_index_feed import KvIndexFeed
            from infera_b200.kv.publisher import KvIndexPublisher

            feed = KvIndexFeed(worker_id(args), args.served_model_name or args.model, getattr(args, "_compat", ""),
                               args.page_size, sink=KvIndexPublisher(args.kv_index_endpoint))
            eng.attach_kv_index(feed)
        aeng = AsyncEngine(eng)
        aeng.start()
        flushers = [p for p in (pub, feed) if p is not None]
        flusher = asyncio.create_task(_flush_loop(*flushers)) if flushers else None

        async def shutdown():
            aeng.stop()
            if flusher is not None:
                flusher.cancel()
            if pub is not None:
                pub.close()

        return aeng, eng.model_cfg.vocab, shutdown
    import subprocess

    from infera_b200.engine.core_ipc import EngineCoreClient, ipc_pair

    proc = None
    if args.attach_core:
        in_addr, out_addr = args.attach_core.split(",")
        client = EngineCoreClient(in_addr, out_addr)
        # the core drops a reply sent before this client's receive socket is
        # connected: ask again until one arrives
        t0 = asyncio.get_running_loop().time()
        while True:
            try:
                await client.call("ping", timeout=1.0)
                break
            except asyncio.TimeoutError:
                if asyncio.get_running_loop().time() - t0 > 120:
                    raise RuntimeError(f"engine core at {in_addr} does not answer")
        st = await client.call("stats")
        info = {"vocab": None, "num_pages": st.get("num_pages")}
        client.mark_ready(info)
    else:
        in_addr, out_addr = ipc_pair()
        client = EngineCoreClient(in_addr, out_addr)
        client._ensure_started()
        proc = subprocess.Popen(_core_cmd(args, in_addr, out_addr))
        while True:
            try:
                info = await client.wait_ready(timeout=5.0)
                break
            except asyncio.TimeoutError:
                if proc.poll() is not None:
                    raise RuntimeError(f"engine core exited with code {proc.returncode}")

    async def shutdown():
        if proc is not None:
            await client.shutdown()
            for _ in range(300):
                if proc.poll() is not None:
                    break
                await asyncio.sleep(0.1)
            if proc.poll() is None:
                proc.terminate()
        client.stop()

    vocab = info.get("vocab")
    if vocab is None:
        from infera_b200.models.config import get_config

        vocab = get_config(args.model).vocab
    return client, vocab, shutdown


async def run_worker(args) -> None:
    import uvicorn

    from infera_b200.engine.server import build_worker_app
    from infera_b200.utils.tokenizer import load_tokenizer

    if args.disagg_mode != "mixed":
        from infera_b200.common.disagg_preflight import preflight

        preflight(mode=args.disagg_mode, advertise_host=args.advertise_host or args.host,
                  kv_endpoint=args.kv_push_endpoint, single_node=(args.advertise_host or args.host) in
                  ("127.0.0.1", "localhost", "0.0.0.0"))
    from infera_b200.models.config import get_config

    # the tokenizer's digest is the KV index's compat key, which the engine
    # core stamps on its index events: load it before the core starts
    tok = load_tokenizer(args.tokenizer, vocab_size=get_config(args.model).vocab)
    args._compat = tok.digest()
    aeng, vocab, shutdown_engine = await start_engine(args)
    app = build_worker_app(aeng, tok, args.served_model_name or args.model)
    server = uvicorn.Server(uvicorn.Config(app, host=args.host, port=args.port, log_level="warning",
                                           access_log=False))
    serve_task = asyncio.create_task(server.serve())
    while not server.started:
        await asyncio.sleep(0.05)
    payload = build_payload(args, tok)
    bus_srv = bus = relay = None
    if args.nats_url:
        from infera_b200.common.nats_wire import NatsBus
        from infera_b200.common.request_transport import BusRequestClient, BusRequestServer, local_http_handler

        bus = await NatsBus(args.nats_url, name=payload["worker_id"]).connect()

        class _W:
            worker_id = payload["worker_id"]

        bus_srv = BusRequestServer(bus, BusRequestClient.token(_W), local_http_handler(f"http://127.0.0.1:{args.port}"),
                                   jetstream=args.nats_jetstream)
        await bus_srv.start()
        if args.kv_events_endpoint:   # KV events onto the bus as well
            from infera_b200.kv.nats_relay import KvEventNatsRelay

            relay = KvEventNatsRelay(bus, payload["worker_id"], args.kv_events_endpoint,
                                     jetstream=args.nats_jetstream, block_size=args.page_size)
            relay.start()
    reg = None
    hb = None
    if args.etcd_endpoint:
        from infera_b200.common.registration import EtcdRegistration

        reg = EtcdRegistration(args.etcd_endpoint, payload)
        await reg.register()
        hb = asyncio.create_task(reg.heartbeat_loop())
    elif args.k8s_register:
        from infera_b200.common.k8s_client import InClusterClient
        from infera_b200.common.registration_k8s import K8sRegistration

        reg = K8sRegistration(InClusterClient(), payload)
        await reg.register()
        hb = asyncio.create_task(reg.heartbeat_loop())
    logger.info("worker %s serving %s", payload["worker_id"], payload["model_name"])
    stop = asyncio.Event()
    loop = asyncio.get_running_loop()
    for sig in (signal.SIGTERM, signal.SIGINT):
        loop.add_signal_handler(sig, stop.set)
    await stop.wait()
    # shutdown: heartbeat off -> deregister -> drain -> stop
    if hb is not None:
        hb.cancel()
    if reg is not None:
        await reg.deregister()
    if bus_srv is not None:   # NATS streams drain (and hand back) like the HTTP ones
        await bus_srv.drain(args.drain_timeout, args.handback_after)
        await bus_srv.stop()
    clean = await aeng.drain(args.drain_timeout, args.handback_after)
    logger.info("drain %s (inflight=%d)", "clean" if clean else "timed out", aeng.inflight)
    await shutdown_engine()
    server.should_exit = True
    await serve_task
    if reg is not None:
        await reg.close()
    if relay is not None:
        await relay.stop()
    if bus is not None:
        await bus.close()


async def _flush_loop(*pubs) -> None:
    while True:
        await asyncio.sleep(0.01)
        for p in pubs:
            p.flush()


def main(argv=None) -> None:
    args = parse_args(argv)
    logging.basicConfig(level=getattr(logging, args.log_level.upper(), logging.INFO))
    asyncio.run(run_worker(args))


if __name__ == "__main__":
    main()

"""Engine core behind ZMQ IPC: the GPU loop and the HTTP front end in
separate processes.

The process that owns the GPU runs :class:`EngineCoreServer`, a tight loop
(drain inbound commands -> one engine step -> push that step's outputs)
with no HTTP, JSON or asyncio work on it. The HTTP server runs in another
process and talks to it through :class:`EngineCoreClient`, which has the
same interface as :class:`infera_b200.engine.async_engine.AsyncEngine`, so
``build_worker_app`` serves either. This keeps the Python interpreter lock
of the serving process away from the engine's step loop: token latency is
the engine's, not the engine's plus the HTTP server's.

Wire (msgpack over two PUSH/PULL pairs; prompt ids travel as int32 bytes):

  client -> core   ["add", rid, ids_i32, sampling dict] | ["abort", rid]
                   | ["handback"] | ["rpc", call_id, name, args] | ["shutdown"]
  core -> client   ["ready", info] | ["out", [[rid, new_ids, finished,
                   reason, n_prompt, n_cached, n_out], ...]]
                   | ["reply", call_id, result]

Reference parity: the reference's workers are stock vLLM / SGLang servers,
whose API server and engine core are likewise separate processes
(``infera/engine/vllm/__main__.py`` launches ``vllm serve``); the engine
here is this framework's own.
"""

from __future__ import annotations

import asyncio
import dataclasses
import os
import time
import uuid

import msgpack
import numpy as np

from infera_b200.engine.async_engine import HANDBACK as HANDBACK_SENTINEL
from infera_b200.engine.request import RequestOutput, SamplingParams

HANDBACK_REASON = "handback"


def ipc_pair(tag: str | None = None) -> tuple[str, str]:
    """Two fresh ``ipc://`` addresses (commands in, outputs out)."""
    t = tag or uuid.uuid4().hex[:12]
    base = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"infera-b200-core-{os.getpid()}-{t}")
    return f"ipc://{base}.in", f"ipc://{base}.out"


def _pack(obj) -> bytes:
    return msgpack.packb(obj, use_bin_type=True)


def _unpack(b: bytes):
    return msgpack.unpackb(b, raw=False)


# ---------------------------------------------------------------------------
# engine side
# ---------------------------------------------------------------------------


class EngineCoreServer:
    """Drives an :class:`LLMEngine` from ZMQ commands. ``run()`` blocks."""

    def __init__(self, engine, in_addr: str, out_addr: str, publisher=None, info: dict | None = None,
                 index_feed=None):
        import zmq

        self.engine = engine
        self.publisher = publisher
        self.index_feed = index_feed
        self.info = dict(info or {})
        self._ctx = zmq.Context.instance()
        self._pull = self._ctx.socket(zmq.PULL)
        self._pull.bind(in_addr)
        self._push = self._ctx.socket(zmq.PUSH)
        self._push.setsockopt(zmq.SNDHWM, 0)
        # with no client connected a PUSH send would block: give up after 2 s
        self._push.setsockopt(zmq.SNDTIMEO, 2000)
        self._push.bind(out_addr)
        self._zmq = zmq
        self._stop = False
        self.dropped = 0
        self._profiler = None
        self.errors = 0
        self.last_error: str | None = None
        self.steps = 0

    # ------------------------------------------------------------------ commands
    def _send(self, obj) -> bool:
        try:
            self._push.send(_pack(obj), copy=False)
            return True
        except self._zmq.Again:
            self.dropped += 1
            return False

    def _send_outputs(self, outs: list[RequestOutput]) -> None:
        if not outs:
            return
        rows = [[o.request_id, o.new_token_ids, o.finished, o.finish_reason, o.num_prompt_tokens,
                 o.num_cached_tokens, o.num_output_tokens] for o in outs]
        self._send(["out", rows])

    def _apply(self, msg) -> None:
        op = msg[0]
        if op == "add":
            _, rid, ids_b, spd = msg
            try:
                ids = np.frombuffer(ids_b, dtype=np.int32).tolist()
                self.engine.add_request(rid, ids, SamplingParams(**spd))
            except Exception as e:
                self._send_outputs([RequestOutput(rid, [], True, f"error: {e}")])
        elif op == "abort":
            if self.engine.abort_request(msg[1]):
                self._send_outputs([RequestOutput(msg[1], [], True, "abort")])
        elif op == "handback":
            outs = []
            for rid in list(self.engine.requests):
                if self.engine.abort_request(rid):
                    outs.append(RequestOutput(rid, [], True, HANDBACK_REASON))
            self._send_outputs(outs)
        elif op == "rpc":
            _, cid, name, args = msg
            try:
                res = self._rpc(name, args)
            except Exception as e:
                res = {"error": repr(e)}
            self._send(["reply", cid, res])
        elif op == "shutdown":
            self._stop = True

    def _rpc(self, name: str, args):
        eng = self.engine
        if name == "stats":
            s = eng.stats()
            s["core_errors"] = self.errors
            s["last_error"] = self.last_error
            return s
        if name == "kv_snapshot":
            return {"block_size": eng.bm.page_size, "block_hashes": [str(h) for h in eng.bm.cached_hashes()],
                    "ts": time.time()}
        if name == "kv_index_snapshot":
            if self.index_feed is None:
                return {"error": "no KV index feed"}
            return self.index_feed.snapshot()
        if name == "profile_start":
            import torch

            if self._profiler is not None:
                return {"error": "already profiling"}
            acts = [torch.profiler.ProfilerActivity.CPU]
            if torch.cuda.is_available():
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self._profiler = torch.profiler.profile(activities=acts, record_shapes=False)
            self._profiler.__enter__()
            eng.trace_phases = True
            return {"status": "started"}
        if name == "profile_stop":
            if self._profiler is None:
                return {"error": "not profiling"}
            p, self._profiler = self._profiler, None
            eng.trace_phases = False
            p.__exit__(None, None, None)
            path = (args or {}).get("path") or f"/tmp/infera_b200_profile_{int(time.time())}.json"
            p.export_chrome_trace(path)
            return {"status": "stopped", "trace": path}
        if name == "ping":
            return {"ok": True}
        raise ValueError(f"unknown rpc {name}")

    def _drain_inbox(self) -> None:
        zmq = self._zmq
        while True:
            try:
                b = self._pull.recv(flags=zmq.NOBLOCK)
            except zmq.Again:
                return
            self._apply(_unpack(b))

    # ------------------------------------------------------------------ loop
    def announce_ready(self, timeout: float = 120.0) -> bool:
        """Tell the client that spawned this core that the engine is up."""
        t0 = time.monotonic()
        while time.monotonic() - t0 < timeout:
            if self._send(["ready", self.info]):
                return True
        return False

    def run_once(self, idle_wait_ms: int = 20) -> bool:
        """One pass: commands, then one engine step if there is work.
        Returns False once a shutdown was received."""
        eng = self.engine
        if not eng.has_unfinished():
            if self._pull.poll(idle_wait_ms):
                self._drain_inbox()
            elif hasattr(eng, "idle"):
                eng.idle()
        else:
            self._drain_inbox()
        if eng.has_unfinished():
            try:
                outs = eng.step()
                self.steps += 1
            except Exception as e:  # keep serving; fail what was in flight
                self.errors += 1
                self.last_error = repr(e)
                outs = []
                for rid in list(eng.requests):
                    if eng.abort_request(rid):
                        outs.append(RequestOutput(rid, [], True, f"error: {e}"))
            self._send_outputs(outs)
        if self.publisher is not None:
            self.publisher.flush()
        if self.index_feed is not None:
            self.index_feed.flush()
        return not self._stop

    def run(self, should_stop=None) -> None:
        dev = getattr(getattr(self.engine, "engine", self.engine), "device", None)
        if dev is not None and dev.type == "cuda":
            import torch

            torch.cuda.set_device(dev)  # per-thread state: this loop may run on a fresh thread
        while self.run_once():
            if should_stop is not None and should_stop():
                break

    def close(self) -> None:
        self._pull.close(linger=0)
        self._push.close(linger=0)


# ---------------------------------------------------------------------------
# HTTP-process side
# ---------------------------------------------------------------------------


class EngineCoreClient:
    """asyncio client with :class:`AsyncEngine`'s serving interface."""

    def __init__(self, in_addr: str, out_addr: str):
        self.in_addr = in_addr
        self.out_addr = out_addr
        self.streams: dict[str, asyncio.Queue] = {}
        self.inflight = 0
        self.draining = False
        self.errors = 0
        self.last_error: str | None = None
        self.info: dict | None = None
        self._rpcs: dict[int, asyncio.Future] = {}
        self._next_call = 0
        self._ready: asyncio.Event | None = None
        self._task: asyncio.Task | None = None
        self._push = None
        self._pull = None
        self._last_stats: dict = {}

    def _ensure_started(self) -> None:
        if self._task is not None:
            return
        import zmq
        import zmq.asyncio

        ctx = zmq.asyncio.Context.instance()
        self._push = ctx.socket(zmq.PUSH)
        self._push.setsockopt(zmq.SNDHWM, 0)
        self._push.connect(self.in_addr)
        self._pull = ctx.socket(zmq.PULL)
        self._pull.connect(self.out_addr)
        self._ready = asyncio.Event()
        self._task = asyncio.get_running_loop().create_task(self._recv_loop())

    async def _recv_loop(self) -> None:
        while True:
            msg = _unpack(await self._pull.recv())
            kind = msg[0]
            if kind == "out":
                for rid, new, fin, reason, npr, nca, nout in msg[1]:
                    q = self.streams.get(rid)
                    if q is None:
                        continue
                    if fin and reason == HANDBACK_REASON:
                        q.put_nowait(HANDBACK_SENTINEL)
                    else:
                        if fin and reason and reason.startswith("error"):
                            self.errors += 1
                            self.last_error = reason
                        q.put_nowait(RequestOutput(rid, new, fin, reason, npr, nca, nout))
                    if fin:
                        if self.streams.pop(rid, None) is not None:
                            self.inflight -= 1
            elif kind == "reply":
                fut = self._rpcs.pop(msg[1], None)
                if fut is not None and not fut.done():
                    fut.set_result(msg[2])
            elif kind == "ready":
                self.info = msg[1]
                self._ready.set()

    async def wait_ready(self, timeout: float = 1800.0) -> dict:
        self._ensure_started()
        await asyncio.wait_for(self._ready.wait(), timeout)
        return self.info or {}

    def mark_ready(self, info: dict | None = None) -> None:
        """For a core that was already running (and announced) before this
        client connected."""
        self._ensure_started()
        self.info = info or {}
        self._ready.set()

    async def call(self, name: str, args=None, timeout: float = 30.0):
        self._ensure_started()
        cid = self._next_call
        self._next_call += 1
        fut = asyncio.get_running_loop().create_future()
        self._rpcs[cid] = fut
        await self._push.send(_pack(["rpc", cid, name, args]))
        try:
            return await asyncio.wait_for(fut, timeout)
        finally:
            self._rpcs.pop(cid, None)

    # ------------------------------------------------------------------ serving API
    async def generate(self, rid: str, prompt_ids: list[int], sp: SamplingParams):
        if self.draining:
            raise RuntimeError("worker is draining")
        self._ensure_started()
        q: asyncio.Queue = asyncio.Queue()
        self.streams[rid] = q
        self.inflight += 1
        ids_b = np.asarray(prompt_ids, dtype=np.int32).tobytes()
        await self._push.send(_pack(["add", rid, ids_b, dataclasses.asdict(sp)]))
        try:
            while True:
                item = await q.get()
                yield item
                if item is HANDBACK_SENTINEL or item.finished:
                    return
        finally:
            if self.streams.pop(rid, None) is not None:  # client went away
                self.inflight -= 1
                await self._push.send(_pack(["abort", rid]))

    def abort(self, rid: str) -> None:
        self._ensure_started()
        asyncio.get_running_loop().create_task(self._push.send(_pack(["abort", rid])))

    def begin_drain(self) -> None:
        self.draining = True

    async def drain(self, timeout: float = 30.0, handback_after: float | None = None) -> bool:
        self.begin_drain()
        t0 = time.monotonic()
        handed = False
        while self.inflight > 0:
            el = time.monotonic() - t0
            if handback_after is not None and el >= handback_after and not handed:
                self._ensure_started()
                await self._push.send(_pack(["handback"]))
                handed = True
            if el >= timeout:
                return False
            await asyncio.sleep(0.02)
        return True

    async def stats_async(self) -> dict:
        try:
            s = await self.call("stats", timeout=5.0)
            self._last_stats = s
        except asyncio.TimeoutError:
            s = dict(self._last_stats)
        s = dict(s)
        s["inflight"] = self.inflight
        s["draining"] = self.draining
        s["errors"] = self.errors + int(s.get("core_errors", 0))
        if s.get("last_error") and not self.last_error:
            self.last_error = s["last_error"]
        return s

    async def kv_snapshot(self) -> dict:
        return await self.call("kv_snapshot")

    async def kv_index_snapshot(self) -> dict:
        return await self.call("kv_index_snapshot")

    async def start_profile(self) -> dict:
        return await self.call("profile_start")

    async def stop_profile(self) -> dict:
        return await self.call("profile_stop", timeout=120.0)

    async def shutdown(self) -> None:
        self._ensure_started()
        await self._push.send(_pack(["shutdown"]))

    def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
        for s in (self._push, self._pull):
            if s is not None:
                s.close(linger=0)


# ---------------------------------------------------------------------------
# engine-core process entry point
# ---------------------------------------------------------------------------


def make_index_feed(a, page_size: int):
    """The tier-aware KV index feed of ``--kv-index-endpoint`` (or None)."""
    if not getattr(a, "kv_index_endpoint", None):
        return None
    from infera_b200.engine.kv_index_feed import KvIndexFeed
    from infera_b200.kv.publisher import KvIndexPublisher

    return KvIndexFeed(a.kv_index_publisher, a.kv_index_model or a.model, a.kv_index_compat, page_size,
                       sink=KvIndexPublisher(a.kv_index_endpoint))


def main(argv=None) -> None:
    """``python -m infera_b200.engine.core_ipc --in ADDR --out ADDR [engine flags]``"""
    import argparse
    import signal

    p = argparse.ArgumentParser(prog="python -m infera_b200.engine.core_ipc")
    p.add_argument("--in", dest="in_addr", required=True)
    p.add_argument("--out", dest="out_addr", required=True)
    p.add_argument("--model", default="llama-3.1-8b")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--max-num-seqs", type=int, default=128)
    p.add_argument("--max-batched-tokens", type=int, default=2048)
    p.add_argument("--mixed-prefill-tokens", type=int, default=256,
                   help="prompt tokens per step while sequences are decoding (0: no cap)")
    p.add_argument("--gpu-memory-utilization", type=float, default=0.90)
    p.add_argument("--num-pages", type=int, default=None)
    p.add_argument("--no-cuda-graphs", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-events-endpoint", default=None)
    p.add_argument("--kv-index-endpoint", default=None,
                   help="ZMQ PUB bind address of the tier-aware KV index events (topic kv-index)")
    p.add_argument("--kv-index-publisher", default="", help="publisher id in those events (the worker id)")
    p.add_argument("--kv-index-model", default="", help="served model name in those events")
    p.add_argument("--kv-index-compat", default="", help="compat key (tokenizer digest) in those events")
    p.add_argument("--kv-tier", default=None)
    p.add_argument("--tp-size", type=int, default=1, help="tensor-parallel ranks (RANK / LOCAL_RANK / MASTER_* from env)")
    p.add_argument("--first-device", type=int, default=0, help="tensor-parallel rank r runs on cuda:(first + r)")
    p.add_argument("--disagg-mode", choices=("mixed", "prefill", "decode"), default="mixed")
    p.add_argument("--kv-push-endpoint", default=None)
    p.add_argument("--dp-attention-size", type=int, default=1,
                   help="data-parallel attention ranks sharing expert-parallel MoE layers (one core per rank; "
                        "'{rank}' in --in / --out is replaced by the rank)")
    p.add_argument("--ep-fused", action="store_true", help="NVLink peer-store expert all-to-all (GPUs)")
    a = p.parse_args(argv)
    if a.dp_attention_size > 1:
        return _main_dp(a)
    from infera_b200.engine.kv_events import KvEventPublisher
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine

    tp = None
    rank = 0
    device = a.device
    if a.tp_size > 1:
        from infera_b200.parallel.launch import init_tp

        tp, rank, device = init_tp(a.tp_size, model=a.model, first_device=a.first_device)
    pub = KvEventPublisher(a.kv_events_endpoint) if a.kv_events_endpoint and rank == 0 else None
    cfg = EngineConfig(model=a.model, page_size=a.page_size, max_num_seqs=a.max_num_seqs,
                       max_batched_tokens=a.max_batched_tokens, gpu_memory_utilization=a.gpu_memory_utilization,
                       mixed_prefill_tokens=a.mixed_prefill_tokens,
                       num_pages=a.num_pages, use_cuda_graphs=not a.no_cuda_graphs, seed=a.seed, kv_tier=a.kv_tier,
                       disagg_mode=a.disagg_mode, kv_push_endpoint=a.kv_push_endpoint)
    eng = LLMEngine(cfg, device=device, event_sink=pub, tp=tp)
    feed = make_index_feed(a, cfg.page_size) if rank == 0 else None
    if feed is not None:
        eng.attach_kv_index(feed)
    if rank > 0:
        from infera_b200.engine.tp_engine import follower_loop

        follower_loop(eng, tp.gloo)
        eng.close()
        tp.close()
        return
    served = eng
    if tp is not None:
        from infera_b200.engine.tp_engine import TPLeader

        served = TPLeader(eng, tp.gloo)
    srv = EngineCoreServer(served, a.in_addr, a.out_addr, publisher=pub,
                           info={"vocab": eng.model_cfg.vocab, "page_size": cfg.page_size,
                                 "num_pages": eng.bm.num_pages, "pid": os.getpid(), "tp_size": a.tp_size},
                           index_feed=feed)
    stop = [False]
    signal.signal(signal.SIGTERM, lambda *_: stop.__setitem__(0, True))
    srv.announce_ready()
    srv.run(should_stop=lambda: stop[0])
    if tp is not None:
        served.shutdown()
        eng.close()
        tp.close()
    if pub is not None:
        pub.close()
    srv.close()


def _main_dp(a) -> None:
    """One data-parallel-attention rank (launched by torch.distributed.run)."""
    import signal
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from infera_b200.engine.dp_attention import DPAttentionEngine, DPServed, EPSpec
    from infera_b200.engine.kv_events import KvEventPublisher
    from infera_b200.engine.llm_engine import EngineConfig

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(a.dp_attention_size)))
    if world != a.dp_attention_size:
        raise SystemExit(f"WORLD_SIZE={world} but --dp-attention-size {a.dp_attention_size}")
    on_gpu = a.device.startswith("cuda")
    if on_gpu:
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", str(rank))))
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    else:
        device = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=600))
    events = a.kv_events_endpoint.format(rank=rank) if a.kv_events_endpoint else None
    pub = KvEventPublisher(events) if events else None
    cfg = EngineConfig(model=a.model, page_size=a.page_size, max_num_seqs=a.max_num_seqs,
                       max_batched_tokens=a.max_batched_tokens, gpu_memory_utilization=a.gpu_memory_utilization,
                       mixed_prefill_tokens=a.mixed_prefill_tokens,
                       num_pages=a.num_pages, use_cuda_graphs=False, seed=a.seed)
    dp = DPAttentionEngine(cfg, EPSpec(rank, world, group=None, gloo=gloo, fused=a.ep_fused and on_gpu),
                           device=device)
    if pub is not None:
        dp.engine.set_event_sink(pub)
    served = DPServed(dp)
    srv = EngineCoreServer(served, a.in_addr.format(rank=rank), a.out_addr.format(rank=rank), publisher=pub,
                           info={"vocab": dp.engine.model_cfg.vocab, "page_size": cfg.page_size,
                                 "num_pages": dp.engine.bm.num_pages, "pid": os.getpid(), "dp_rank": rank,
                                 "dp_size": world})
    # SIGTERM ends the loop on the next vote of every rank: a rank that
    # stopped alone would leave the others waiting in the collective
    stop = [False]
    signal.signal(signal.SIGTERM, lambda *_: stop.__setitem__(0, True))
    srv.announce_ready()

    def should_stop():
        t = torch.tensor([1 if (stop[0] or srv._stop) else 0], dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=gloo)
        return bool(t.item())

    # every pass: one lockstep step vote (inside run_once) and one stop vote
    while True:
        srv.run_once()
        if should_stop():
            break
    for lw in dp.engine.model.w.layers:
        if "moe" in lw and hasattr(lw["moe"], "close"):
            lw["moe"].close()
    if pub is not None:
        pub.close()
    srv.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

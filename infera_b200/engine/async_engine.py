"""Runs :class:`LLMEngine` on a dedicated thread for asyncio servers.

Requests enter through a thread-safe inbox; every engine iteration's
outputs are pushed to the owning request's asyncio queue with
``call_soon_threadsafe``. The in-flight count is exact (admitted and not yet
finished), which is what drain waits on.

Drain: ``begin_drain()`` refuses new requests; ``drain(timeout)`` waits for
in-flight work to finish, and after ``handback_after`` seconds hands the
still-running requests back (their streams end with the draining notice, so
the router migrates them).
"""

from __future__ import annotations

import asyncio
import queue
import threading
import time
from dataclasses import dataclass

from infera_b200.engine.request import RequestOutput, SamplingParams


@dataclass
class _Stream:
    loop: asyncio.AbstractEventLoop
    q: asyncio.Queue


HANDBACK = "handback"


class AsyncEngine:
    def __init__(self, engine):
        self.engine = engine
        self.inbox: queue.Queue = queue.Queue()
        self.streams: dict[str, _Stream] = {}
        self._lock = threading.Lock()
        self._thread: threading.Thread | None = None
        self._running = False
        self.draining = False
        self.inflight = 0
        self.errors = 0
        self.last_error: str | None = None
        self.profiler = None

    # ------------------------------------------------------------------ loop
    def start(self) -> None:
        self._running = True
        self._thread = threading.Thread(target=self._loop, name="engine-loop", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._running = False
        self.inbox.put(("noop", None))
        if self._thread is not None:
            self._thread.join(timeout=30)

    def _deliver(self, rid: str, item) -> None:
        st = self.streams.get(rid)
        if st is not None:
            st.loop.call_soon_threadsafe(st.q.put_nowait, item)

    def _apply(self, op, arg) -> None:
        if op == "add":
            rid, ids, sp = arg
            try:
                self.engine.add_request(rid, ids, sp)
            except Exception as e:
                self._finish_stream(rid, RequestOutput(rid, [], True, f"error: {e}"))
        elif op == "abort":
            if self.engine.abort_request(arg):
                self._finish_stream(arg, RequestOutput(arg, [], True, "abort"))
        elif op == "handback":
            for rid in list(self.streams):
                if self.engine.abort_request(rid):
                    self._finish_stream(rid, HANDBACK)

    def _finish_stream(self, rid: str, item) -> None:
        self._deliver(rid, item)
        with self._lock:
            if self.streams.pop(rid, None) is not None:
                self.inflight -= 1

    def _loop(self) -> None:
        dev = getattr(self.engine, "device", None)
        if dev is not None and dev.type == "cuda":
            import torch

            torch.cuda.set_device(dev)  # the CUDA current device is per thread
        while self._running:
            try:
                block = not self.engine.has_unfinished()
                while True:
                    try:
                        op, arg = self.inbox.get(block=block, timeout=0.05 if block else 0)
                    except queue.Empty:
                        break
                    self._apply(op, arg)
                    block = False
                if not self.engine.has_unfinished():
                    continue
                for o in self.engine.step():
                    if o.finished:
                        self._finish_stream(o.request_id, o)
                    else:
                        self._deliver(o.request_id, o)
            except Exception as e:  # keep serving; fail the affected requests
                self.errors += 1
                self.last_error = repr(e)
                for rid in list(self.streams):
                    self.engine.abort_request(rid)
                    self._finish_stream(rid, RequestOutput(rid, [], True, f"error: {e}"))

    # ------------------------------------------------------------------ API
    async def generate(self, rid: str, prompt_ids: list[int], sp: SamplingParams):
        """Async iterator of RequestOutput (or HANDBACK when the worker
        hands the request back during drain)."""
        if self.draining:
            raise RuntimeError("worker is draining")
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        with self._lock:
            self.streams[rid] = _Stream(loop, q)
            self.inflight += 1
        self.inbox.put(("add", (rid, prompt_ids, sp)))
        try:
            while True:
                item = await q.get()
                yield item
                if item is HANDBACK or item.finished:
                    return
        finally:
            if rid in self.streams:  # client went away
                self.inbox.put(("abort", rid))

    def abort(self, rid: str) -> None:
        self.inbox.put(("abort", rid))

    def begin_drain(self) -> None:
        self.draining = True

    async def drain(self, timeout: float = 30.0, handback_after: float | None = None) -> bool:
        """Wait until nothing is in flight. Returns True if drained cleanly."""
        self.begin_drain()
        t0 = time.monotonic()
        handed = False
        while self.inflight > 0:
            el = time.monotonic() - t0
            if handback_after is not None and el >= handback_after and not handed:
                self.inbox.put(("handback", None))
                handed = True
            if el >= timeout:
                return False
            await asyncio.sleep(0.02)
        return True

    def stats(self) -> dict:
        s = self.engine.stats()
        s["inflight"] = self.inflight
        s["draining"] = self.draining
        s["errors"] = self.errors
        return s

    async def stats_async(self) -> dict:
        return self.stats()

    async def kv_snapshot(self) -> dict:
        bm = self.engine.bm
        return {"block_size": bm.page_size, "block_hashes": [str(h) for h in bm.cached_hashes()], "ts": time.time()}

    async def kv_index_snapshot(self) -> dict:
        feed = getattr(self.engine, "kv_index", None)
        if feed is None:
            return {"error": "no KV index feed"}
        return feed.snapshot()

    async def start_profile(self) -> dict:
        import torch

        if self.profiler is not None:
            return {"error": "already profiling"}
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self.profiler = torch.profiler.profile(activities=acts, record_shapes=False)
        self.profiler.__enter__()
        self.engine.trace_phases = True
        return {"status": "started"}

    async def stop_profile(self) -> dict:
        if self.profiler is None:
            return {"error": "not profiling"}
        p, self.profiler = self.profiler, None
        self.engine.trace_phases = False
        p.__exit__(None, None, None)
        path = f"/tmp/infera_b200_profile_{int(time.time())}.json"
        try:
            p.export_chrome_trace(path)
        except Exception as e:
            return {"status": "stopped", "error": str(e)}
        return {"status": "stopped", "trace": path}

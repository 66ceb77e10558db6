"""Engine core behind ZMQ IPC: the client gives the same tokens as the
in-process engine, hand-back and RPCs work, and the worker CLI runs its
engine core as a child process (tiny model on CPU)."""

import asyncio
import os
import signal
import subprocess
import sys
import threading
import time

import httpx

from infera_b200.engine.async_engine import HANDBACK
from infera_b200.engine.core_ipc import EngineCoreClient, EngineCoreServer, ipc_pair
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _engine():
    return LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=128), device="cpu")


def test_client_matches_in_process_engine():
    prompts = [[5, 6, 7, 8, 9], list(range(100, 140))]
    ref = _engine().generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))
    in_addr, out_addr = ipc_pair()
    srv = EngineCoreServer(_engine(), in_addr, out_addr)
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()

    async def go():
        cl = EngineCoreClient(in_addr, out_addr)
        cl.mark_ready()

        async def one(i, p):
            toks = []
            async for o in cl.generate(f"r{i}", p, SamplingParams(max_tokens=5, ignore_eos=True)):
                toks.extend(o.new_token_ids)
            return toks

        outs = await asyncio.gather(*(one(i, p) for i, p in enumerate(prompts)))
        st = await cl.stats_async()
        snap = await cl.kv_snapshot()
        assert cl.inflight == 0
        await cl.shutdown()
        cl.stop()
        return outs, st, snap

    outs, st, snap = asyncio.run(go())
    th.join(timeout=10)
    assert outs == ref
    assert st["finished"] == 2 and st["generation_tokens"] == 10
    assert snap["block_size"] == 16 and len(snap["block_hashes"]) >= 2


def test_handback_and_bad_request():
    in_addr, out_addr = ipc_pair()
    srv = EngineCoreServer(_engine(), in_addr, out_addr)
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()

    async def go():
        cl = EngineCoreClient(in_addr, out_addr)
        cl.mark_ready()
        got = []

        async def long_one():
            async for o in cl.generate("long", list(range(50)), SamplingParams(max_tokens=10_000, ignore_eos=True)):
                got.append(o)
                if o is HANDBACK:
                    return

        bad = [o async for o in cl.generate("bad", [], SamplingParams())]
        t = asyncio.create_task(long_one())
        await asyncio.sleep(0.5)
        assert cl.inflight == 1
        ok = await cl.drain(timeout=10.0, handback_after=0.1)
        await t
        refused = False
        try:
            async for _ in cl.generate("late", [1, 2], SamplingParams()):
                pass
        except RuntimeError:
            refused = True
        await cl.shutdown()
        cl.stop()
        return ok, got, bad, refused

    ok, got, bad, refused = asyncio.run(go())
    th.join(timeout=10)
    assert ok and got[-1] is HANDBACK
    assert bad[-1].finished and bad[-1].finish_reason.startswith("error")
    assert refused  # a draining client refuses new work before it reaches the core


def test_worker_cli_spawns_engine_core():
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    port = 18977
    p = subprocess.Popen([sys.executable, "-m", "infera_b200.engine.worker", "--model", "tiny-dense", "--device", "cpu",
                          "--no-cuda-graphs", "--num-pages", "128", "--port", str(port), "--drain-timeout", "5"],
                         env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, start_new_session=True)
    try:
        t0 = time.time()
        up = False
        while time.time() - t0 < 120 and p.poll() is None:
            try:
                if httpx.get(f"http://127.0.0.1:{port}/health", timeout=2).status_code == 200:
                    up = True
                    break
            except httpx.HTTPError:
                time.sleep(0.3)
        assert up, p.stdout.read().decode()[-3000:] if p.poll() is not None else "worker did not come up"
        r = httpx.post(f"http://127.0.0.1:{port}/v1/completions",
                       json={"model": "tiny-dense", "prompt": [1, 2, 3, 4], "max_tokens": 4, "ignore_eos": True,
                             "return_token_ids": True}, timeout=60)
        assert r.status_code == 200 and len(r.json()["choices"][0]["token_ids"]) == 4
        m = httpx.get(f"http://127.0.0.1:{port}/metrics", timeout=10).text
        assert "infera_engine:generation_tokens_total" in m
        # busy-time counters: steps that ran a forward and the time inside them
        vals = {ln.split()[0].split("{")[0]: float(ln.split()[-1]) for ln in m.splitlines()
                if ln.startswith("infera_engine:")}
        assert vals.get("infera_engine:steps_total", 0) >= 4
        assert vals.get("infera_engine:forward_seconds_total", 0) > 0
        p.send_signal(signal.SIGTERM)
        assert p.wait(timeout=60) == 0
    finally:
        if p.poll() is None:
            os.killpg(p.pid, signal.SIGKILL)

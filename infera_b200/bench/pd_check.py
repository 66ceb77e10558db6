"""Prefill/decode disaggregation end to end on two GPUs of one node.

    python -m infera_b200.bench.pd_check [--model llama-3.1-8b] [--requests 16] [--prompt-len 2048]

Starts the etcd stand-in, the native router, a prefill worker on cuda:0 and
a decode worker on cuda:1 (both see both GPUs: the prefill engine maps the
decode engine's KV cache with CUDA IPC and pushes pages over NVLink), sends
concurrent streamed requests through the router, and prints one JSON line:
completions, errors, TTFT percentiles, the decode instance's prompt tokens
computed (only the last token of each prompt when the push worked), and
the push bandwidth from the prefill instance's counters (bytes pushed over
the push kernels' device time, CUDA events around each launch) against
the 770 GB/s NVLink reference.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import random
import subprocess
import sys
import time

import httpx

from infera_b200.bench.e2e import _spawn, _stop, _wait_http, router_cmd
from infera_b200.common.engine_metrics import parse_exposition
from infera_b200.common.net import free_tcp_port

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _worker(model, device, mode, port, etcd, kv_ep, logdir, events_port):
    cmd = [sys.executable, "-m", "infera_b200.engine.worker", "--model", model, "--served-model-name", model,
           "--device", device, "--disagg-mode", mode, "--port", str(port), "--host", "127.0.0.1",
           "--etcd-endpoint", f"127.0.0.1:{etcd}", "--kv-events-endpoint", f"tcp://127.0.0.1:{events_port}",
           "--max-num-seqs", "64", "--log-level", "warning"]
    if kv_ep:
        cmd += ["--kv-push-endpoint", kv_ep]
    return _spawn(cmd, os.path.join(logdir, f"pd_{mode}.log"))


async def _one(c, url, model, prompt, n):
    t0 = time.monotonic()
    first = None
    toks = 0
    async with c.stream("POST", url + "/v1/completions", json={"model": model, "prompt": prompt, "max_tokens": n,
                                                                "stream": True, "ignore_eos": True,
                                                                "return_token_ids": True}) as r:
        if r.status_code != 200:
            return None
        async for line in r.aiter_lines():
            if not line.startswith("data:") or "[DONE]" in line:
                continue
            obj = json.loads(line[5:])
            if obj.get("error"):
                return None
            for ch in obj.get("choices") or []:
                k = len(ch.get("token_ids") or [])
                if k and first is None:
                    first = time.monotonic() - t0
                toks += k
    return first, toks


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--requests", type=int, default=16)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--max-tokens", type=int, default=32)
    a = ap.parse_args(argv)
    logdir = os.environ.get("INFERA_LOG_DIR", "/tmp")   # worker / router logs
    etcd, router = free_tcp_port(), free_tcp_port()
    pport, dport = free_tcp_port(), free_tcp_port()
    kv_ep = f"ipc:///tmp/infera-b200-pd-{os.getpid()}"
    procs = []
    try:
        procs.append(_spawn([sys.executable, "-m", "infera_b200.common.etcd_fake", "--port", str(etcd)],
                            os.path.join(logdir, "pd_etcd.log")))
        _wait_http(f"http://127.0.0.1:{etcd}/health", lambda r: True, 60)
        procs.append(_spawn(router_cmd("native", etcd, router), os.path.join(logdir, "pd_router.log")))
        procs.append(_worker(a.model, "cuda:1", "decode", dport, etcd, kv_ep, logdir, free_tcp_port()))
        procs.append(_worker(a.model, "cuda:0", "prefill", pport, etcd, None, logdir, free_tcp_port()))
        url = f"http://127.0.0.1:{router}"
        if not _wait_http(url + "/v1/workers", lambda r: len(r.json().get("workers", [])) >= 2, 600):
            raise SystemExit("PD workers did not register")
        rng = random.Random(0)
        prompts = [[rng.randrange(1000, 120000) for _ in range(a.prompt_len)] for _ in range(a.requests)]

        async def go():
            async with httpx.AsyncClient(timeout=httpx.Timeout(600.0)) as c:
                await _one(c, url, a.model, prompts[0][:64], 2)  # warm-up
                t0 = time.monotonic()
                res = await asyncio.gather(*(_one(c, url, a.model, p, a.max_tokens) for p in prompts))
                wall = time.monotonic() - t0
                pm = parse_exposition((await c.get(f"http://127.0.0.1:{pport}/metrics")).text)
                dm = parse_exposition((await c.get(f"http://127.0.0.1:{dport}/metrics")).text)
            return res, wall, pm, dm

        res, wall, pm, dm = asyncio.run(go())
        ok = [r for r in res if r is not None and r[1] == a.max_tokens]
        ttft = sorted(r[0] for r in ok if r[0] is not None)
        pb = pm.get("infera_engine:pd_push_bytes_total", 0.0)
        ps = pm.get("infera_engine:pd_push_device_seconds_total", 0.0)
        out = {"model": a.model, "requests": a.requests, "prompt_len": a.prompt_len, "completed": len(ok),
               "errors": a.requests - len(ok), "wall_s": round(wall, 3),
               "ttft_p50_s": round(ttft[len(ttft) // 2], 4) if ttft else None,
               "ttft_max_s": round(ttft[-1], 4) if ttft else None,
               "pushes": pm.get("infera_engine:pd_pushes_total"), "push_gbytes": round(pb / 1e9, 3),
               "push_gbs_device": round(pb / ps / 1e9, 1) if ps else None,
               "push_frac_of_nvlink_770": round(pb / ps / 770e9, 3) if ps else None,
               "decode_prompt_tokens_computed": dm.get("infera_engine:prompt_tokens_total"),
               "prefill_prompt_tokens_computed": pm.get("infera_engine:prompt_tokens_total")}
        print(json.dumps(out), flush=True)
    finally:
        for p in reversed(procs):
            _stop(p)


if __name__ == "__main__":
    main()

"""End-to-end measurement through the public HTTP API.

The engine that served the device-timed window is wrapped in the worker's
OpenAI-compatible server (the same app ``python -m infera_b200.engine.worker``
serves) on ``127.0.0.1:<port>``, and a separate load-generator process
replays the trace against ``/v1/completions`` (streamed). Latencies are the
client's wall clock; every engine iteration copies its packed inputs from
pinned host memory and reads the sampled ids back, and those bytes are
counted from the engine's copy counters over the timed slices.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import threading
import time

from infera_b200.bench.slo import SLO, ReqRecord, percentile, summarize


def _serve_in_thread(app, port: int):
    import uvicorn

    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning",
                                           access_log=False))
    th = threading.Thread(target=server.run, name="e2e-http", daemon=True)
    th.start()
    t0 = time.time()
    while not server.started and time.time() - t0 < 30:
        time.sleep(0.05)
    return server, th


def run_e2e_on_engine(engine, *, model: str, rank: int, sessions: range, rate: float, warmup_s: float,
                      timed_s: float, seed: int) -> dict:
    from infera_b200.engine.async_engine import AsyncEngine
    from infera_b200.engine.server import build_worker_app
    from infera_b200.utils.tokenizer import load_tokenizer

    port = 18100 + rank
    aeng = AsyncEngine(engine)
    aeng.start()
    app = build_worker_app(aeng, load_tokenizer(None, vocab_size=engine.model_cfg.vocab), model)
    server, th = _serve_in_thread(app, port)
    h2d0, d2h0 = engine.runner.h2d_bytes, engine.runner.d2h_bytes
    it0 = engine.num_steps
    cmd = [sys.executable, "-m", "infera_b200.bench.http_loadgen", "--url", f"http://127.0.0.1:{port}",
           "--model", model, "--sessions", f"{sessions.start}:{sessions.stop}", "--rate", str(rate),
           "--duration", str(warmup_s + timed_s), "--seed", str(seed + 1000), "--drain-s", "0"]
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.getcwd(), env.get("PYTHONPATH", "")])
    out = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env, timeout=warmup_s + timed_s + 300)
    h2d, d2h = engine.runner.h2d_bytes - h2d0, engine.runner.d2h_bytes - d2h0
    iters = engine.num_steps - it0
    server.should_exit = True
    th.join(timeout=10)
    aeng.stop()
    if out.returncode != 0:
        raise RuntimeError(f"load generator failed: {out.stderr.decode()[-2000:]}")
    res = json.loads(out.stdout)
    recs = []
    for r in res["records"]:
        rec = ReqRecord("", r["arrival"], prompt_len=r["prompt_len"], cached_len=r["cached_len"],
                        out_len=r["out_len"])
        rec.token_times = r["token_times"]
        rec.first_token = rec.token_times[0] if rec.token_times else None
        rec.finish = r["finish"]
        recs.append(rec)
    win = (warmup_s, warmup_s + timed_s)
    st = summarize(recs, win, SLO())
    done = [r for r in recs if r.finish is not None and win[0] <= r.finish <= win[1]]
    total = warmup_s + timed_s
    return {
        "window_s": timed_s, "slo_met": st["slo_met"], "completed": st["completed"],
        "ttfts": [r.ttft for r in done if r.ttft is not None], "itls": [x for r in done for x in r.itls()],
        "errors": res["errors"],
        # copies happen every engine iteration; report them per benchmark step (1 s slice)
        "h2d_per_step": h2d / total, "d2h_per_step": d2h / total, "iterations": iters,
    }


def aggregate(allr: list[dict]) -> dict:
    win = max(r["window_s"] for r in allr)
    ttfts = [x for r in allr for x in r["ttfts"]]
    itls = [x for r in allr for x in r["itls"]]
    return {
        "value": round(sum(r["slo_met"] for r in allr) / win, 4),
        "unit": "req/s",
        "path": "OpenAI /v1/completions over HTTP (streamed), client wall clock",
        "completed": sum(r["completed"] for r in allr),
        "slo_met": sum(r["slo_met"] for r in allr),
        "ttft_p50_s": round(percentile(ttfts, 50), 4),
        "ttft_p99_s": round(percentile(ttfts, 99), 4),
        "itl_p99_ms": round(1000 * percentile(itls, 99), 3),
        "errors": sum(r["errors"] for r in allr),
        "h2d_bytes_per_step": int(sum(r["h2d_per_step"] for r in allr)),
        "d2h_bytes_per_step": int(sum(r["d2h_per_step"] for r in allr)),
    }

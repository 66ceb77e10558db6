"""Prefill-decode disaggregated serving of the agentic PD trace, end to end,
on one box: 1 prefill instance + 1 decode instance, each tensor-parallel
over ``--tp`` GPUs (prefill on GPUs 0..tp-1, decode on tp..2tp-1), behind
the KV-aware router, the prompt's KV pushed layer by layer over NVLink.

    python -m infera_b200.bench.pd_fleet [--model llama-3.1-70b] [--tp 4] [--rate 1.0]
        [--warmup 20] [--duration 60] [--tail 60]

Every process is this framework's public entry point: the etcd stand-in,
``python -m infera_b200.server`` (native router), two ``python -m
infera_b200.engine.worker --tp-size N`` workers (each launches its engine
core ranks with torch.distributed.run). The load generator replays the
``pd-70b`` trace (input 8k-32k tokens with 90% shared-prefix reuse across
turns, 256 output tokens) at ``--rate`` requests/s against the router's
``/v1/completions`` (streamed), after an untimed prewarm of every shared
prefix. Goodput counts the requests that arrive in the timed window and
finish within the SLO (TTFT <= ``--ttft-slo`` s, ITL p99 <= 50 ms). Prints
one JSON line: goodput, TTFT / ITL percentiles, and the KV push's bytes and
device-timed bandwidth from the prefill instance's counters against the
NVLink link (900 GB/s nominal, 770 GB/s measured peer copy).
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import sys
import time

import httpx

from infera_b200.bench.e2e import _spawn, _stop, _wait_http, router_cmd
from infera_b200.bench.slo import SLO, ReqRecord, cohort, percentile, summarize
from infera_b200.common.engine_metrics import parse_exposition
from infera_b200.common.net import free_tcp_port


def _worker(a, mode: str, first: int, port: int, etcd: int, kv_ep: str | None, logdir: str):
    cmd = [sys.executable, "-m", "infera_b200.engine.worker", "--model", a.model, "--served-model-name", a.model,
           "--tp-size", str(a.tp), "--first-device", str(first), "--device", f"cuda:{first}",
           "--disagg-mode", mode, "--port", str(port), "--host", "127.0.0.1",
           "--etcd-endpoint", f"127.0.0.1:{etcd}", "--kv-events-endpoint", f"tcp://127.0.0.1:{free_tcp_port()}",
           "--max-num-seqs", str(a.max_num_seqs), "--max-batched-tokens", str(a.max_batched_tokens),
           "--log-level", "warning"]
    if kv_ep:
        cmd += ["--kv-push-endpoint", kv_ep]
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "0"))
    return _spawn(cmd, os.path.join(logdir, f"pd_fleet_{mode}.log"), env=env)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-70b")
    ap.add_argument("--tp", type=int, default=4)
    ap.add_argument("--rate", type=float, default=1.0)
    ap.add_argument("--warmup", type=float, default=20.0)
    ap.add_argument("--duration", type=float, default=60.0)
    ap.add_argument("--tail", type=float, default=60.0)
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-batched-tokens", type=int, default=4096)
    ap.add_argument("--ttft-slo", type=float, default=10.0)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    logdir = os.environ.get("INFERA_LOG_DIR", "/tmp")
    etcd, router = free_tcp_port(), free_tcp_port()
    pport, dport = free_tcp_port(), free_tcp_port()
    kv_ep = f"ipc:///tmp/infera-b200-pd-fleet-{os.getpid()}"
    procs = []
    t_setup = time.time()
    try:
        procs.append(_spawn([sys.executable, "-m", "infera_b200.common.etcd_fake", "--port", str(etcd)],
                            os.path.join(logdir, "pd_fleet_etcd.log")))
        _wait_http(f"http://127.0.0.1:{etcd}/health", lambda r: True, 60)
        procs.append(_spawn(router_cmd("native", etcd, router), os.path.join(logdir, "pd_fleet_router.log")))
        procs.append(_worker(a, "decode", a.tp, dport, etcd, kv_ep, logdir))
        procs.append(_worker(a, "prefill", 0, pport, etcd, None, logdir))
        url = f"http://127.0.0.1:{router}"
        if not _wait_http(url + "/v1/workers", lambda r: len(r.json().get("workers", [])) >= 2, 1500):
            raise SystemExit("PD workers did not register (see pd_fleet_*.log)")
        setup_s = time.time() - t_setup
        from infera_b200.bench.http_loadgen import prewarm
        from infera_b200.bench.http_loadgen import run as loadgen

        sids = list(range(a.sessions))
        pw = asyncio.run(prewarm(url, a.model, "pd-70b", sids, a.seed, extra=2, extra_len=2048, timeout=1200.0))
        res = asyncio.run(loadgen(url, a.model, "pd-70b", sids, a.rate, a.warmup + a.duration + a.tail, a.seed,
                                  stop_after_s=0.0))
        recs = []
        for r in res["records"]:
            rec = ReqRecord("", r["arrival"], prompt_len=r["prompt_len"], cached_len=r["cached_len"],
                            out_len=r["out_len"])
            rec.token_times = r["token_times"]
            rec.first_token = rec.token_times[0] if rec.token_times else None
            rec.finish = r["finish"]
            recs.append(rec)
        win = (a.warmup, a.warmup + a.duration)
        slo = SLO(ttft_s=a.ttft_slo)
        st = summarize(recs, win, slo)
        done = cohort(recs, win)
        ttfts = [r.ttft for r in done if r.ttft is not None]
        itls = [x for r in done for x in r.itls()]

        async def metrics():
            async with httpx.AsyncClient(timeout=30) as c:
                pm = parse_exposition((await c.get(f"http://127.0.0.1:{pport}/metrics")).text)
                dm = parse_exposition((await c.get(f"http://127.0.0.1:{dport}/metrics")).text)
            return pm, dm

        pm, dm = asyncio.run(metrics())
        pb = pm.get("infera_engine:pd_push_bytes_total", 0.0)
        ps = pm.get("infera_engine:pd_push_device_seconds_total", 0.0)
        out = {
            "metric": "goodput req/s within p99 TTFT/ITL SLO on the PD trace; p50 TTFT",
            "model": a.model, "placement": f"prefill TP{a.tp} on GPUs 0-{a.tp - 1}, decode TP{a.tp} on GPUs "
                                          f"{a.tp}-{2 * a.tp - 1}", "rate": a.rate,
            "window_s": a.duration, "goodput_rps": round(st["goodput_rps"], 4), "arrived": st["cohort"],
            "completed": st["completed"], "slo_met": st["slo_met"], "slo": {"ttft_s": a.ttft_slo, "itl_p99_ms": 50},
            "ttft_p50_s": round(percentile(ttfts, 50), 4) if ttfts else None,
            "ttft_p99_s": round(percentile(ttfts, 99), 4) if ttfts else None,
            "itl_p50_ms": round(1000 * percentile(itls, 50), 3) if itls else None,
            "itl_p99_ms": round(1000 * percentile(itls, 99), 3) if itls else None,
            "prefix_hit_rate": round(st["prefix_hit_rate"], 4), "errors": res["errors"],
            "prewarm": pw, "setup_s": round(setup_s, 1),
            "pushes": pm.get("infera_engine:pd_pushes_total"), "push_gbytes": round(pb / 1e9, 3),
            "push_gbs_device": round(pb / ps / 1e9, 1) if ps else None,
            "push_frac_of_nvlink_900": round(pb / ps / 900e9, 3) if ps else None,
            "push_frac_of_measured_770": round(pb / ps / 770e9, 3) if ps else None,
            "decode_prompt_tokens_computed": dm.get("infera_engine:prompt_tokens_total"),
            "prefill_prompt_tokens_computed": pm.get("infera_engine:prompt_tokens_total"),
            # busy time and rate of each instance: low busy time points at
            # admission / hand-off, a low rate inside the forwards at compute
            "prefill_steps": pm.get("infera_engine:steps_total"),
            "prefill_forward_s": pm.get("infera_engine:forward_seconds_total"),
            "prefill_tokens_per_forward_s": round(pm.get("infera_engine:prompt_tokens_total", 0.0)
                                                  / pm["infera_engine:forward_seconds_total"], 1)
            if pm.get("infera_engine:forward_seconds_total") else None,
            "decode_steps": dm.get("infera_engine:steps_total"),
            "decode_forward_s": dm.get("infera_engine:forward_seconds_total"),
        }
        print(json.dumps(out), flush=True)
    finally:
        for p in reversed(procs):
            _stop(p)


if __name__ == "__main__":
    main()

"""End-to-end measurement through the public HTTP API, behind the router.

The same fleet shape as the reference arm: one worker per GPU, all behind
one KV-aware router that discovers them through etcd (an in-memory etcd v3
JSON-gateway server; no etcd binary exists here) and follows their KV
events over ZMQ. Per rank:

* the engine that served the device-timed window is wrapped in an
  :class:`~infera_b200.engine.core_ipc.EngineCoreServer` whose step loop
  runs on a thread of the benchmark process (the GPU owner), with its
  prefix cache cleared first so the run starts cold like the reference's;
* ``python -m infera_b200.engine.worker --attach-core`` serves the
  OpenAI-compatible HTTP API for it in a separate process and registers it;
* rank 0 also runs the router (``python -m infera_b200.server``) and the
  etcd stand-in;
* a separate load-generator process replays the trace - the same sessions
  and seed as the reference arm - against the router's ``/v1/completions``
  (streamed). Latencies are the client's wall clock.

Every engine iteration copies its packed inputs from pinned host memory and
reads the sampled ids back; those bytes are counted from the engine's copy
counters over the run.
"""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
import threading
import time

from infera_b200.bench.slo import SLO, ReqRecord, cohort, percentile, summarize

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
ETCD_PORT = 23890
ROUTER_PORT = 28100
WORKER_PORT0 = 29200
EVENTS_PORT0 = 29300


def _spawn(cmd, log_path, env=None):
    f = open(log_path, "w")
    e = dict(env or os.environ)
    e["PYTHONPATH"] = os.pathsep.join([ROOT] + [p for p in e.get("PYTHONPATH", "").split(os.pathsep) if p])
    return subprocess.Popen(cmd, stdout=f, stderr=subprocess.STDOUT, env=e, start_new_session=True)


def _stop(p, sig=signal.SIGTERM, timeout=60.0):
    if p is None or p.poll() is not None:
        return
    try:
        os.killpg(p.pid, sig)
        p.wait(timeout=timeout)
    except Exception:
        try:
            os.killpg(p.pid, signal.SIGKILL)
        except Exception:
            pass


def _wait_http(url: str, pred, timeout: float) -> bool:
    import httpx

    t0 = time.time()
    while time.time() - t0 < timeout:
        try:
            r = httpx.get(url, timeout=5)
            if r.status_code == 200 and pred(r):
                return True
        except Exception:
            pass
        time.sleep(0.5)
    return False


def router_cmd(backend: str, etcd_port: int = ETCD_PORT, router_port: int = ROUTER_PORT) -> list[str]:
    return [sys.executable, "-m", "infera_b200.server", "--discovery-backend", "etcd",
            "--etcd-endpoint", f"127.0.0.1:{etcd_port}", "--router-policy", "kv-aware",
            "--router-backend", backend, "--host", "127.0.0.1", "--port", str(router_port),
            "--log-level", os.environ.get("INFERA_E2E_LOG_LEVEL", "warning")]


def run_e2e_fleet(engine, *, model: str, rank: int, world: int, barrier, sessions: range, rate: float,
                  warmup_s: float, timed_s: float, seed: int, router_backend: str = "python",
                  logdir: str | None = None, trace: str = "agentic-8b", drain_s: float = 0.0,
                  ports: dict | None = None, appear_timeout: float = 300.0, tail_s: float = 0.0,
                  prewarm: bool = True) -> dict:
    """``barrier()`` synchronises the ranks (host-side). ``ports`` overrides
    the fixed ports (keys etcd, router, worker0, events0). Arrivals continue
    for ``tail_s`` after the timed window so that the window's arrivals can
    finish under the same load; ``prewarm``: the untimed warm-up of
    :func:`infera_b200.bench.http_loadgen.prewarm` before the trace clock."""
    P = {"etcd": ETCD_PORT, "router": ROUTER_PORT, "worker0": WORKER_PORT0, "events0": EVENTS_PORT0}
    P.update(ports or {})
    from infera_b200.engine.core_ipc import EngineCoreServer, ipc_pair
    from infera_b200.engine.kv_events import KvEventPublisher

    logdir = logdir or os.environ.get("INFERA_LOG_DIR", "/tmp")   # worker / router logs
    procs = []
    th = None
    stop = threading.Event()
    worker = None
    pub = None
    try:
        if rank == 0:
            procs.append(_spawn([sys.executable, "-m", "infera_b200.common.etcd_fake", "--port", str(P["etcd"])],
                                os.path.join(logdir, "e2e_etcd.log")))
            _wait_http(f"http://127.0.0.1:{P['etcd']}/health", lambda r: True, 60)
            procs.append(_spawn(router_cmd(router_backend, P["etcd"], P["router"]),
                                os.path.join(logdir, "e2e_router.log")))
        barrier()
        # cold start: nothing cached from the device-timed window
        ev_ep = f"tcp://127.0.0.1:{P['events0'] + rank}"
        pub = KvEventPublisher(ev_ep)
        engine.set_event_sink(pub)
        engine.bm.clear_cache()
        in_addr, out_addr = ipc_pair(f"r{rank}")
        srv = EngineCoreServer(engine, in_addr, out_addr, publisher=pub)
        th = threading.Thread(target=srv.run, kwargs={"should_stop": stop.is_set}, name="engine-core",
                              daemon=True)
        th.start()
        port = P["worker0"] + rank
        worker = _spawn([sys.executable, "-m", "infera_b200.engine.worker", "--attach-core", f"{in_addr},{out_addr}",
                         "--model", model, "--served-model-name", model, "--host", "127.0.0.1", "--port", str(port),
                         "--etcd-endpoint", f"127.0.0.1:{P['etcd']}", "--kv-events-endpoint", ev_ep,
                         "--page-size", str(engine.bm.page_size), "--log-level", os.environ.get("INFERA_E2E_LOG_LEVEL", "warning")],
                        os.path.join(logdir, f"e2e_worker{rank}.log"))
        if rank == 0:
            ok = _wait_http(f"http://127.0.0.1:{P['router']}/v1/workers",
                            lambda r: len(r.json().get("workers", [])) >= world, appear_timeout)
            if not ok:
                raise RuntimeError("e2e: workers did not appear at the router")
        barrier()
        h2d0, d2h0 = engine.runner.h2d_bytes, engine.runner.d2h_bytes
        it0 = engine.num_steps
        cmd = [sys.executable, "-m", "infera_b200.bench.http_loadgen", "--url", f"http://127.0.0.1:{P['router']}",
               "--model", model, "--sessions", f"{sessions.start}:{sessions.stop}", "--rate", str(rate),
               "--duration", str(warmup_s + timed_s + tail_s), "--seed", str(seed), "--drain-s", str(drain_s),
               "--trace", trace] + (["--prewarm"] if prewarm else [])
        env = dict(os.environ)
        env["PYTHONPATH"] = os.pathsep.join([ROOT, env.get("PYTHONPATH", "")])
        out = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env,
                             timeout=warmup_s + timed_s + tail_s + 900)
        h2d, d2h = engine.runner.h2d_bytes - h2d0, engine.runner.d2h_bytes - d2h0
        iters = engine.num_steps - it0
        if out.returncode != 0:
            raise RuntimeError(f"load generator failed: {out.stderr.decode()[-2000:]}")
        res = json.loads(out.stdout)
        barrier()
    finally:
        _stop(worker)
        stop.set()
        if th is not None:
            th.join(timeout=120)
        for p in reversed(procs):
            _stop(p)
        engine.set_event_sink(None)
        if pub is not None:
            pub.close()
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
    done = cohort(recs, win)
    total = warmup_s + timed_s + tail_s
    return {
        "window_s": timed_s, "slo_met": st["slo_met"], "completed": st["completed"], "cohort": st["cohort"],
        "prewarm": res.get("prewarm"),
        "ttfts": [r.ttft for r in done if r.ttft is not None], "itls": [x for r in done for x in r.itls()],
        "errors": res["errors"], "prefix_hit_rate": st["prefix_hit_rate"],
        # copies happen every engine iteration; report them per benchmark step (1 s slice)
        "h2d_per_step": h2d / total, "d2h_per_step": d2h / total, "iterations": iters,
    }


def aggregate(allr: list[dict], path: str) -> dict:
    win = max(r["window_s"] for r in allr)
    ttfts = [x for r in allr for x in r["ttfts"]]
    itls = [x for r in allr for x in r["itls"]]
    return {
        "value": round(sum(r["slo_met"] for r in allr) / win, 4),
        "unit": "req/s",
        "path": path,
        "arrived": sum(r.get("cohort", r["completed"]) for r in allr),
        "completed": sum(r["completed"] for r in allr),
        "slo_met": sum(r["slo_met"] for r in allr),
        "ttft_p50_s": round(percentile(ttfts, 50), 4),
        "ttft_p99_s": round(percentile(ttfts, 99), 4),
        "itl_p50_ms": round(1000 * percentile(itls, 50), 3),
        "itl_p99_ms": round(1000 * percentile(itls, 99), 3),
        "errors": sum(r["errors"] for r in allr),
        "prefix_hit_rate": round(sum(r.get("prefix_hit_rate", 0.0) for r in allr) / len(allr), 4),
        "h2d_bytes_per_step": int(sum(r["h2d_per_step"] for r in allr)),
        "d2h_bytes_per_step": int(sum(r["d2h_per_step"] for r in allr)),
    }

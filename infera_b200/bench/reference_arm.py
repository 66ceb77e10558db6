"""Reference arm of the serving benchmark.

Runs the UNMODIFIED reference (installed under ``baseline/_ref``) through its
own public API and stock launchers, for the same metric, model shape and
trace as this framework's arm:

* ``python -m infera.engine.vllm`` - one stock worker per GPU: the
  reference's launcher spawns ``vllm serve`` (vLLM from the image) on a
  Llama-3.1-8B-shaped model directory with ``--load-format dummy`` (random
  weights), registers it in etcd and publishes KV events over ZMQ;
* ``python -m infera.server`` - the reference router (KV-aware policy, etcd
  discovery, HTTP request transport, ZMQ KV events);
* the same seeded trace, replayed against the router's ``/v1/completions``
  by the HTTP load generator (prompts as ``t<id>`` words, which the
  generated word-level tokenizer maps to exactly the trace's token ids).

The reference discovers workers only through etcd or Kubernetes; no etcd
binary exists here, so an in-memory server speaking the etcd v3 JSON gateway
API (``infera_b200.common.etcd_fake``) stands in for etcd. Nothing else on
the path is this framework's code. Timing is the client's wall clock (the
reference runs in separate engine processes and exposes no device timer).
"""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
ETCD_PORT = 23790
ROUTER_PORT = 28000
WORKER_PORT0 = 29100
MODEL_DIR = "/tmp/infera_ref_model"
SERVED = "llama-3.1-8b"


def _log(*a):
    if int(os.environ.get("RANK", "0")) == 0:
        print("[reference]", *a, file=sys.stderr, flush=True)


def _env(local_rank: int | None = None) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([REF_DIR] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    env["HF_HUB_OFFLINE"] = "1"
    env["TRANSFORMERS_OFFLINE"] = "1"
    env["VLLM_NO_USAGE_STATS"] = "1"
    env["DO_NOT_TRACK"] = "1"
    if local_rank is not None:
        env["CUDA_VISIBLE_DEVICES"] = str(local_rank)
    return env


def _spawn(cmd, env, log_path):
    f = open(log_path, "w")
    return subprocess.Popen(cmd, env=env, stdout=f, stderr=subprocess.STDOUT, start_new_session=True)


def _kill(p):
    if p is None or p.poll() is not None:
        return
    try:
        os.killpg(p.pid, signal.SIGTERM)
        p.wait(timeout=30)
    except Exception:
        try:
            os.killpg(p.pid, signal.SIGKILL)
        except Exception:
            pass


def _wait_workers(n: int, timeout: float) -> bool:
    import httpx

    t0 = time.time()
    while time.time() - t0 < timeout:
        try:
            r = httpx.get(f"http://127.0.0.1:{ROUTER_PORT}/v1/workers", timeout=5)
            if r.status_code == 200 and len(r.json().get("workers", [])) >= n:
                return True
        except Exception:
            pass
        time.sleep(2)
    return False


def run_reference(args) -> dict:
    if not os.path.isdir(os.path.join(REF_DIR, "infera")):
        return {"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}
    try:
        import vllm  # noqa: F401
    except Exception as e:
        return {"impl": "reference", "unavailable": f"vLLM (the reference's CUDA backend) not importable: {e}"}
    import asyncio

    import torch.distributed as dist

    from infera_b200.bench.e2e import aggregate
    from infera_b200.bench.hf_model_dir import write_model_dir
    from infera_b200.bench.http_loadgen import prewarm
    from infera_b200.bench.http_loadgen import run as loadgen
    from infera_b200.bench.slo import SLO, ReqRecord, cohort, summarize

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        dist.init_process_group("gloo", timeout=timedelta(seconds=1800))

    def barrier():
        if world > 1:
            dist.barrier()

    logdir = os.environ.get("INFERA_LOG_DIR", "/tmp")   # worker / router logs
    procs = []
    t_setup = time.time()
    try:
        if rank == 0:
            write_model_dir(MODEL_DIR, args.model)
            procs.append(_spawn([sys.executable, "-m", "infera_b200.common.etcd_fake", "--port", str(ETCD_PORT)],
                                dict(os.environ), os.path.join(logdir, "ref_etcd.log")))
        barrier()
        worker_cmd = [sys.executable, "-m", "infera.engine.vllm", "--discovery-backend", "etcd",
                      "--etcd-endpoint", f"127.0.0.1:{ETCD_PORT}", "--request-transport", "http",
                      "--kv-event-transport", "zmq", "--model", MODEL_DIR, "--served-model-name", SERVED,
                      "--load-format", "dummy", "--max-model-len", "33792", "--host", "127.0.0.1",
                      "--port", str(WORKER_PORT0 + rank), "--block-size", "16", "--gpu-memory-utilization", "0.90",
                      "--max-num-seqs", str(args.max_num_seqs), "--seed", str(args.seed)]
        procs.append(_spawn(worker_cmd, _env(local), os.path.join(logdir, f"ref_worker{rank}.log")))
        if rank == 0:
            router_cmd = [sys.executable, "-m", "infera.server", "--discovery-backend", "etcd",
                          "--etcd-endpoint", f"127.0.0.1:{ETCD_PORT}", "--request-transport", "http",
                          "--kv-event-transport", "zmq", "--router-policy", "kv-aware",
                          "--router-tokenizer-path", MODEL_DIR, "--host", "127.0.0.1", "--port", str(ROUTER_PORT)]
            procs.append(_spawn(router_cmd, _env(None), os.path.join(logdir, "ref_router.log")))
        ok = _wait_workers(world, timeout=1500) if rank == 0 else True
        if world > 1:
            flag = [ok]
            dist.broadcast_object_list(flag, src=0)
            ok = flag[0]
        if not ok:
            return {"impl": "reference", "unavailable": "reference workers did not register within 25 min "
                                                         "(see ref_worker*.log / ref_router.log)"}
        _log(f"fleet up after {time.time() - t_setup:.0f}s")
        barrier()
        url = f"http://127.0.0.1:{ROUTER_PORT}"
        base = rank * 64
        warm = args.warmup * args.slice
        timed = args.steps * args.slice
        tail = args.tail
        sids = list(range(base, base + 64))
        # the same untimed warm-up as this framework's end-to-end arm
        pw = asyncio.run(prewarm(url, SERVED, "agentic-8b", sids, args.seed + rank, text_prompts=True))
        barrier()
        res = asyncio.run(loadgen(url, SERVED, "agentic-8b", sids, args.rate, warm + timed + tail,
                                  args.seed + rank, stop_after_s=0.0, text_prompts=True))
        recs = []
        for r in res["records"]:
            rec = ReqRecord("", r["arrival"], prompt_len=r["prompt_len"], cached_len=r["cached_len"],
                            out_len=r["out_len"])
            rec.token_times = r["token_times"]
            rec.first_token = rec.token_times[0] if rec.token_times else None
            rec.finish = r["finish"]
            recs.append(rec)
        st = summarize(recs, (warm, warm + timed), SLO())
        done = cohort(recs, (warm, warm + timed))
        local_res = {"window_s": timed, "slo_met": st["slo_met"], "completed": st["completed"], "cohort": st["cohort"],
                     "prewarm": pw,
                     "ttfts": [r.ttft for r in done if r.ttft is not None], "itls": [x for r in done for x in r.itls()],
                     "errors": res["errors"], "h2d_per_step": 0, "d2h_per_step": 0,
                     "output_tok_s": st["output_tok_s"], "prefix_hit_rate": st["prefix_hit_rate"]}
        allr = [local_res]
        if world > 1:
            allr = [None] * world
            dist.all_gather_object(allr, local_res)
        if rank != 0:
            return {}
        agg = aggregate(allr, "reference router /v1/completions over HTTP (streamed), client wall clock")
        # the reference arm is end to end already: its figure is both the
        # value and the e2e entry (prompts go over HTTP as text and every
        # engine step copies its inputs in and its tokens out inside vLLM;
        # those bytes are not observable from outside the reference)
        e2e = dict(agg)
        e2e["h2d_bytes_per_step"] = None
        e2e["d2h_bytes_per_step"] = None
        return {
            "metric": "goodput req/s within p99 TTFT/ITL SLO on synthetic agentic trace; p50 TTFT",
            "value": agg["value"], "unit": "req/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000 * args.slice, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 (stock reference worker: vLLM, fp8 KV cache by default)",
            "data": "synthetic (seeded multi-turn agentic trace, random token ids; random-init weights)",
            "config": {"model": args.model, "deployment": f"{world} stock vLLM worker(s) at TP=1 behind the "
                                                          "reference's KV-aware router",
                       "parallelism": f"dp{world}", "arrival_rate_per_gpu": args.rate, "sessions_per_gpu": 64,
                       "slo": {"ttft_p99_s": 2.0, "itl_p99_ms": 50.0},
                       "step": f"{args.slice:.0f} s slice of the open-loop trace", "timing": "client wall clock",
                       "etcd": "in-memory etcd v3 JSON gateway stand-in",
                       "goodput_cohort": f"requests arriving in the timed window; arrivals continue {tail:g} s "
                                         f"after it for them to finish",
                       "prewarm": "each prefix group's system prefix + 8 random 1024-token prompts, untimed"},
            "ttft_p50_s": agg["ttft_p50_s"], "ttft_p99_s": agg["ttft_p99_s"], "itl_p99_ms": agg["itl_p99_ms"],
            "itl_p50_ms": agg["itl_p50_ms"], "arrived": agg["arrived"],
            "completed": agg["completed"], "slo_met": agg["slo_met"], "errors": agg["errors"],
            "output_tok_s": round(sum(r["output_tok_s"] for r in allr), 1),
            "prefix_hit_rate": round(sum(r["prefix_hit_rate"] for r in allr) / len(allr), 4),
            "setup_s": round(time.time() - t_setup, 1),
            "impl": "reference",
            "e2e": e2e,
        }
    finally:
        for p in reversed(procs):
            _kill(p)
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    from bench import parse_args

    print(json.dumps(run_reference(parse_args(sys.argv[1:]))))

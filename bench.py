"""Serving benchmark: goodput (req/s within the p99 TTFT / ITL SLO) and p50
TTFT on the synthetic multi-turn agentic trace, Llama-3.1-8B-shaped model
(random-init bf16), one engine instance per GPU (TP=1).

    python bench.py --gpus N --steps K --warmup W [--rate R] [--impl ours|reference]

N > 1 is launched with torch.distributed.run (one rank per GPU, NCCL for the
barriers and the final gather). Every rank serves its own 64 sessions (two
prefix groups of 32; at N = 8 that is the full 512-session trace) with
Poisson arrivals at ``--rate`` requests/s per GPU: weak scaling.

One step is a one-second slice of the open-loop trace (the engine iterates
continuously across slices). W warm-up slices run untimed, then K slices
are timed between barrier + synchronize fences. Token timestamps are CUDA
events recorded at the end of each engine iteration, relative to the
window's origin. The goodput cohort is every request that ARRIVED in the
timed window; the trace keeps arriving for ``--tail`` seconds after it
(untimed) so that those requests finish under the same load, and a request
counts once it has finished within the SLO. The value is the sum over ranks
of SLO-meeting requests of the cohort divided by the longest rank's window.
(Counting by arrival keeps the figure independent of where the window's
edges fall relative to a server's latency; both arms use it.)

The end-to-end figure ("e2e") is the reference arm's setup with this
framework's parts: every rank's engine (prefix cache cleared, then the same
untimed prewarm through the router as the reference arm gets) serves the
OpenAI-compatible HTTP API from a separate worker process, all workers sit
behind one KV-aware router (etcd discovery, ZMQ KV events), and each rank's
load generator replays the same sessions and seed as the reference arm
against the router's /v1/completions (streamed), timed by the client's wall
clock. That includes every step's pinned host->device copy of the inputs
and device->host copy of the sampled tokens.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

# stdout carries exactly one JSON line: NCCL's own messages (the version
# banner when NCCL_DEBUG is set) go to stderr
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "goodput req/s within p99 TTFT/ITL SLO on synthetic agentic trace; p50 TTFT"
MODEL = "llama-3.1-8b"
PUBLISHED_BASELINE = None  # the reference publishes no number for this config
SESSIONS_PER_GPU = 64


_T0 = time.time()


def log(*a) -> None:
    """Progress on stderr (stdout carries only the JSON line)."""
    if int(os.environ.get("RANK", "0")) == 0:
        print(f"[bench {time.time() - _T0:7.1f}s]", *a, file=sys.stderr, flush=True)


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=15)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--rate", type=float, default=8.0,
                    help="Poisson arrivals per second per GPU (8 = 64 req/s over 8 instances, the top of the sweep)")
    ap.add_argument("--slice", type=float, default=1.0, help="seconds of trace per step")
    ap.add_argument("--tail", type=float, default=8.0,
                    help="seconds the trace keeps arriving after the timed window, for the window's arrivals "
                         "to finish (the goodput cohort is the requests that arrived in the window)")
    ap.add_argument("--mixed-prefill-tokens", type=int, default=256,
                    help="prompt tokens per engine step while sequences are decoding")
    ap.add_argument("--model", default=MODEL)
    ap.add_argument("--max-num-seqs", type=int, default=128)
    ap.add_argument("--max-batched-tokens", type=int, default=2048)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--router-backend", choices=("python", "native"), default="native",
                    help="router in front of the e2e fleet: the C++ data plane (default) or the Python one")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args(argv)


def _dist_init():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        global _GLOO
        _GLOO = dist.new_group(backend="gloo", timeout=timedelta(seconds=900))
    return rank, world, local


_GLOO = None


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _host_barrier(world):
    """Barrier over a gloo group: no GPU work, safe while another thread of
    this process drives the engine."""
    if world > 1:
        import torch.distributed as dist

        dist.barrier(group=_GLOO)


def _gather(obj, world):
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj, group=_GLOO)
    return out


def run_ours(args) -> dict:
    import torch

    from infera_b200.bench.clocks import ClockSampler
    from infera_b200.bench.replay import EngineReplay
    from infera_b200.bench.slo import SLO, cohort, percentile, summarize
    from infera_b200.bench.trace import PRESETS
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.ops import kernels as K

    rank, world, local = _dist_init()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    spec = PRESETS["agentic-8b"]
    ecfg = EngineConfig(model=args.model, max_num_seqs=args.max_num_seqs,
                        max_batched_tokens=args.max_batched_tokens, use_cuda_graphs=not args.no_graphs,
                        seed=args.seed, mixed_prefill_tokens=args.mixed_prefill_tokens)
    eng = LLMEngine(ecfg, device=dev)
    log(f"engine ready: {eng.bm.num_pages} KV pages, graphs={ecfg.use_cuda_graphs}")
    sessions = list(range(rank * SESSIONS_PER_GPU, (rank + 1) * SESSIONS_PER_GPU))
    rp = EngineReplay(eng, spec, sessions, rate=args.rate, seed=args.seed + rank)
    rp.prime_prefixes()
    torch.cuda.synchronize()
    log("prefixes primed")
    _barrier(world)
    rp.start_clock()
    rp.run_until(args.warmup * args.slice)            # W warm-up slices
    log(f"warm-up done: {eng.num_steps} iterations, running={eng.num_running()} waiting={eng.num_waiting()}")
    # ---- timed window: K slices between barrier + synchronize fences
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    ev_start = torch.cuda.Event(enable_timing=True)
    ev_start.record()
    t_start_host = rp.now()
    launches0 = K.LAUNCHES[0]
    h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
    steps0 = eng.num_steps
    sampler = ClockSampler(gpu_index=local)
    sampler.start()
    rp.run_until(t_start_host + args.steps * args.slice)
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    ev_end = torch.cuda.Event(enable_timing=True)
    ev_end.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches1 = K.LAUNCHES[0]
    h2d1, d2h1 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
    log(f"timed window done: {eng.num_steps - steps0} iterations, running={eng.num_running()} "
        f"waiting={eng.num_waiting()}")
    # the trace keeps arriving while the window's arrivals finish (untimed)
    rp.run_until(rp.now() + args.tail)
    records = rp.resolve()
    w0 = rp.ev0.elapsed_time(ev_start) / 1000.0
    w1 = rp.ev0.elapsed_time(ev_end) / 1000.0
    st = summarize(records, (w0, w1), SLO())
    done = cohort(records, (w0, w1))
    local_res = {
        "window_s": w1 - w0, "slo_met": st["slo_met"], "completed": st["completed"],
        "ttfts": [r.ttft for r in done],
        "itls": [x for r in done for x in r.itls()],
        "out_tokens": st["output_tok_s"] * st["window_s"],
        "launches": launches1 - launches0, "cohort": st["cohort"],
        "engine_steps": eng.num_steps - steps0,
        "h2d": h2d1 - h2d0, "d2h": d2h1 - d2h0,
        "prefix_hit_rate": st["prefix_hit_rate"], "clocks": clocks,
        "kernel_status": K.scratch(dev).read_status(),
        "step_profile": rp.step_profile((w0, w1)),
    }
    e2e_local = None
    if not args.no_e2e:
        from infera_b200.bench.e2e import run_e2e_fleet

        log(f"e2e: {world} worker(s) behind the {args.router_backend} router, load generator per rank")
        e2e_local = run_e2e_fleet(eng, model=args.model, rank=rank, world=world, barrier=lambda: _host_barrier(world),
                                  sessions=range(rank * SESSIONS_PER_GPU, (rank + 1) * SESSIONS_PER_GPU),
                                  rate=args.rate, warmup_s=args.warmup * args.slice,
                                  timed_s=(args.e2e_steps or args.steps) * args.slice, seed=args.seed + rank,
                                  router_backend=args.router_backend, tail_s=args.tail)
        log(f"e2e done: {e2e_local['completed']} completed, {e2e_local['errors']} errors")
    allr = _gather(local_res, world)
    e2e_all = _gather(e2e_local, world) if e2e_local is not None else None
    del rp
    eng_cfg = ecfg
    del eng
    torch.cuda.empty_cache()
    if rank != 0:
        return {}
    win = max(r["window_s"] for r in allr)
    good = sum(r["slo_met"] for r in allr)
    ttfts = [x for r in allr for x in r["ttfts"] if x is not None]
    itls = [x for r in allr for x in r["itls"]]
    res = {
        "value": good / win,
        "window_s": win,
        "arrived": sum(r["cohort"] for r in allr),
        "completed": sum(r["completed"] for r in allr),
        "slo_met": good,
        "ttft_p50_s": percentile(ttfts, 50),
        "ttft_p99_s": percentile(ttfts, 99),
        "itl_p50_ms": 1000 * percentile(itls, 50),
        "itl_p99_ms": 1000 * percentile(itls, 99),
        "output_tok_s": sum(r["out_tokens"] for r in allr) / win,
        "launches": sum(r["launches"] for r in allr),
        "engine_steps": max(r["engine_steps"] for r in allr),
        "h2d": sum(r["h2d"] for r in allr), "d2h": sum(r["d2h"] for r in allr),
        "prefix_hit_rate": sum(r["prefix_hit_rate"] for r in allr) / len(allr),
        "clocks": allr[0]["clocks"],
        "kernel_status": max(r["kernel_status"] for r in allr),
        "step_profile": allr[0]["step_profile"],
        "engine_cfg": {"max_num_seqs": eng_cfg.max_num_seqs, "max_batched_tokens": eng_cfg.max_batched_tokens},
    }
    if e2e_all is not None:
        from infera_b200.bench.e2e import aggregate

        res["e2e"] = aggregate(e2e_all, f"OpenAI /v1/completions over HTTP (streamed) through the "
                                        f"{args.router_backend} KV-aware router, client wall clock")
    return res


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        from infera_b200.bench.reference_arm import run_reference

        line = run_reference(args)
        print(json.dumps(line), flush=True)
        return 0
    t0 = time.time()
    res = run_ours(args)
    rank = int(os.environ.get("RANK", "0"))
    e2e = res.get("e2e")
    if rank != 0:
        return 0
    K_ = args.steps
    line = {
        "metric": METRIC,
        "value": round(res["value"], 4),
        "unit": "req/s",
        "n_gpus": args.gpus,
        "steps": K_,
        "warmup": args.warmup,
        "ms_per_step": round(1000 * res["window_s"] / K_, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None if PUBLISHED_BASELINE is None else round(res["value"] / PUBLISHED_BASELINE, 4),
        "dtype": "bf16",
        "data": "synthetic (seeded multi-turn agentic trace, random token ids; random-init weights)",
        "config": {
            "model": MODEL, "architecture": "32L, hidden 4096, 32q/8kv heads, head_dim 128, SwiGLU 14336, "
                                            "vocab 128256, RoPE theta 500000",
            "deployment": f"{args.gpus} instance(s) at TP=1; device-timed: sessions pinned to instances by "
                          f"prefix group; e2e: behind one KV-aware router",
            "parallelism": f"dp{args.gpus}",
            "global_batch": f"continuous batching, <= {res['engine_cfg']['max_num_seqs']} seqs / instance",
            "seq_len": "context <= 32768 (prefix 4096 shared by 32 sessions, +U[256,1024]/turn, out U[128,512])",
            "arrival_rate_per_gpu": args.rate,
            "sessions_per_gpu": SESSIONS_PER_GPU,
            "slo": {"ttft_p99_s": 2.0, "itl_p99_ms": 50.0},
            "step": f"{args.slice:.0f} s slice of the open-loop trace",
            "l2": "inputs larger than L2 (16 GB of weights + KV read every iteration)",
            "prefixes_primed": True,
            "max_batched_tokens": res["engine_cfg"]["max_batched_tokens"],
            "mixed_prefill_tokens": args.mixed_prefill_tokens,
            "goodput_cohort": f"requests arriving in the timed window; arrivals continue {args.tail:g} s after "
                              f"it (untimed) for them to finish",
            "prewarm": "device-timed: every prefix group's system prefix computed before the clock; e2e: each "
                       "prefix group's system prefix + 8 random 1024-token prompts through the router, untimed "
                       "(the reference arm gets the same)",
        },
        "ttft_p50_s": round(res["ttft_p50_s"], 4),
        "ttft_p99_s": round(res["ttft_p99_s"], 4),
        "itl_p50_ms": round(res["itl_p50_ms"], 3),
        "itl_p99_ms": round(res["itl_p99_ms"], 3),
        "arrived": res["arrived"],
        "completed": res["completed"],
        "slo_met": res["slo_met"],
        "output_tok_s": round(res["output_tok_s"], 1),
        "prefix_hit_rate": round(res["prefix_hit_rate"], 4),
        "engine_iterations": res["engine_steps"],
        "kernel_status": res["kernel_status"],
        "step_profile_rank0": res["step_profile"],
        "clocks": res["clocks"],
        "gpu_launches": res["launches"],
        "impl": "ours",
        "wall_s": round(time.time() - t0, 1),
    }
    if e2e is not None:
        line["e2e"] = e2e
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

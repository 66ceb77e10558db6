"""Kernel-time breakdown of one decode step and one mixed step (a prompt
chunk joining running decodes) of the serving engine.

    python -m infera_b200.bench.step_breakdown [--model llama-3.1-8b] [--decodes 48] [--context 2048]
        [--chunk 224] [--top 15]

Builds the engine, fills it with ``--decodes`` running sequences of
``--context`` cached tokens, then records (torch.profiler, CUDA activity)
one decode-only step and one step in which a ``--chunk``-token prompt joins
them. Prints one JSON line per step kind: the step's wall time, the summed
device time of its kernels, the host time until the step returned, and the
top kernels by device time. Shares, not absolute bench numbers: the
profiler serialises nothing but adds its own overhead to the host side.
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def _top(prof, top: int) -> tuple[float, list[dict]]:
    rows = []
    total = 0.0
    for ev in prof.key_averages():
        dev_us = getattr(ev, "device_time_total", None)
        if dev_us is None:
            dev_us = getattr(ev, "cuda_time_total", 0.0)
        if not dev_us or ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        total += dev_us
        rows.append({"kernel": ev.key[:90], "us": round(dev_us, 1), "calls": ev.count})
    rows.sort(key=lambda r: -r["us"])
    for r in rows:
        r["share"] = round(r["us"] / total, 3) if total else 0.0
    return total, rows[:top]


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--decodes", type=int, default=48)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--chunk", type=int, default=224)
    ap.add_argument("--top", type=int, default=15)
    ap.add_argument("--graphs", type=int, default=1)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--time-steps", type=int, default=0,
                    help="also time this many decode-only steps without the profiler (host clock per step)")
    a = ap.parse_args(argv)

    from torch.profiler import ProfilerActivity, profile

    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams

    eng = LLMEngine(EngineConfig(model=a.model, use_cuda_graphs=bool(a.graphs),
                                 max_num_seqs=max(64, a.decodes + 4)), device=a.device)
    V = eng.model.cfg.vocab
    g = torch.Generator().manual_seed(0)
    sp = SamplingParams(max_tokens=100000, ignore_eos=True)
    for i in range(a.decodes):
        eng.add_request(f"d{i}", torch.randint(0, V, (a.context,), generator=g).tolist(), sp)
    # run until every sequence decodes, then a few decode steps
    for _ in range(10000):
        eng.step()
        if getattr(eng, "last_step_shape", (1, 0))[0] == 0:
            break
    for _ in range(5):
        eng.step()
    dev = eng.device
    sync = (lambda: torch.cuda.synchronize(dev)) if dev.type == "cuda" else (lambda: None)

    def record(kind: str, before=None) -> None:
        if before is not None:
            before()
        sync()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            t0 = time.perf_counter()
            eng.step()
            host = time.perf_counter() - t0
            sync()
            wall = time.perf_counter() - t0
        total, rows = _top(prof, a.top)
        print(json.dumps({"step": kind, "shape": list(getattr(eng, "last_step_shape", (0, 0))),
                          "wall_ms": round(wall * 1e3, 3), "host_return_ms": round(host * 1e3, 3),
                          "device_kernel_ms": round(total / 1e3, 3), "top": rows}), flush=True)

    # warm both shapes once outside the profiler
    eng.step()
    eng.add_request("warm", torch.randint(0, V, (a.chunk,), generator=g).tolist(),
                    SamplingParams(max_tokens=1, ignore_eos=True))
    eng.step()
    eng.step()
    if a.time_steps > 0:
        ts = []
        for _ in range(a.time_steps):
            sync()
            t0 = time.perf_counter()
            eng.step()
            sync()
            ts.append((time.perf_counter() - t0) * 1e3)
        ts.sort()
        print(json.dumps({"step": "decode_timed", "n": len(ts), "p50_ms": round(ts[len(ts) // 2], 3),
                          "min_ms": round(ts[0], 3), "p90_ms": round(ts[int(0.9 * len(ts))], 3)}), flush=True)
    record("decode")
    record("mixed", lambda: eng.add_request("chunk", torch.randint(0, V, (a.chunk,), generator=g).tolist(),
                                            SamplingParams(max_tokens=1, ignore_eos=True)))


if __name__ == "__main__":
    main()

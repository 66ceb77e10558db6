"""Expert-parallel serving of the DeepSeek-V3-shaped MoE with data-parallel
attention: one rank per GPU, each a full engine over its own requests
(MLA attention with all 128 heads, its own latent KV cache), the routed
experts sharded E / world per rank and exchanged through the NVLink
peer-store all-to-all fused with the grouped GEMMs.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m infera_b200.bench.ep_serve [--rate 2.0] [--warmup 20] [--duration 60] [--tail 60]

Every rank replays its share of the ``ep-dsv3`` trace (input 2k-16k random
tokens, output 256-1024) at ``rate / world`` requests/s, Poisson. The ranks
step in lockstep: one host vote per iteration decides whether any rank has
work (a rank without any runs a one-token dummy forward so the expert
exchanges line up) and whether the window is over, so every rank takes the
same collective steps. Token times come from CUDA events on each rank's
stream (clock origin taken after a barrier). Prints one JSON line from rank
0: goodput (requests that arrived in the timed window and met TTFT <=
``--ttft-slo`` and ITL p99 <= ``--itl-slo-ms``), output tokens/s over all
ranks, TTFT / ITL percentiles, idle forwards.

Reference counterpart: the DeepSeek EP recipes the reference launches
through SGLang (``--enable-dp-attention`` + ``--ep-size``, MoRI all-to-all;
``infera/engine/sglang/__main__.py:73-100``).
"""

from __future__ import annotations

import argparse
import json
import os
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from infera_b200.bench.replay import EngineReplay
from infera_b200.bench.slo import SLO, cohort, percentile, summarize
from infera_b200.bench.trace import PRESETS
from infera_b200.ops import kernels as K


class _Lockstep:
    """The DP-attention engine as the replay sees it: ``step`` runs this
    rank's forward, or the dummy forward when it has nothing scheduled; the
    caller has already voted that some rank has work."""

    def __init__(self, dp):
        self.dp = dp
        self.engine = dp.engine
        self.device = dp.engine.device
        self.runner = dp.engine.runner

    def add_request(self, *a, **kw):
        return self.engine.add_request(*a, **kw)

    def has_unfinished(self) -> bool:
        return self.engine.has_unfinished()

    @property
    def last_step_shape(self):
        return getattr(self.engine, "last_step_shape", (0, 0))

    def step(self):
        n0 = self.runner.forwards
        outs = self.engine.step()
        if self.runner.forwards == n0:
            self.runner.idle_forward()
            self.dp.idle_forwards += 1
        return outs


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="deepseek-v3")
    ap.add_argument("--rate", type=float, default=2.0, help="total requests/s over all ranks")
    ap.add_argument("--warmup", type=float, default=20.0)
    ap.add_argument("--duration", type=float, default=60.0)
    ap.add_argument("--tail", type=float, default=60.0)
    ap.add_argument("--sessions-per-rank", type=int, default=32)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-batched-tokens", type=int, default=4096)
    ap.add_argument("--mixed-prefill-tokens", type=int, default=512)
    ap.add_argument("--ttft-slo", type=float, default=10.0)
    ap.add_argument("--itl-slo-ms", type=float, default=50.0)
    ap.add_argument("--nccl-a2a", action="store_true", help="NCCL all-to-all instead of the fused peer-store path")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--trace", default="ep-dsv3")
    ap.add_argument("--cpu", action="store_true", help="gloo ranks on the CPU (host-side logic; tiny model)")
    a = ap.parse_args(argv)

    from infera_b200.engine.dp_attention import DPAttentionEngine, EPSpec
    from infera_b200.engine.llm_engine import EngineConfig

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.cpu:
        device = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    else:
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", str(rank))))
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=300))
    t_init = time.time()
    cfg = EngineConfig(model=a.model, max_num_seqs=a.max_num_seqs, max_batched_tokens=a.max_batched_tokens,
                       mixed_prefill_tokens=a.mixed_prefill_tokens, use_cuda_graphs=False, seed=a.seed)
    dp = DPAttentionEngine(cfg, EPSpec(rank, world, group=None, gloo=gloo, fused=not (a.nccl_a2a or a.cpu)),
                           device=device)
    eng = _Lockstep(dp)
    init_s = time.time() - t_init
    spec = PRESETS[a.trace]
    sids = [rank + world * i for i in range(a.sessions_per_rank)]
    rp = EngineReplay(eng, spec, sids, a.rate / world, seed=a.seed * 100 + rank)
    t_end = a.warmup + a.duration + a.tail
    dist.barrier(group=gloo)
    rp.start_clock()
    iters = 0
    while True:
        rp._admit_arrivals()
        v = torch.tensor([1 if eng.has_unfinished() else 0, 1 if rp.now() >= t_end else 0], dtype=torch.int32)
        dist.all_reduce(v, op=dist.ReduceOp.MAX, group=gloo)
        if v[1]:
            break
        if v[0]:
            rp.step_once()
            iters += 1
        else:
            time.sleep(0.001)
    if not a.cpu:
        torch.cuda.synchronize()
    recs = rp.resolve()
    win = (a.warmup, a.warmup + a.duration)
    slo = SLO(ttft_s=a.ttft_slo, itl_s=a.itl_slo_ms / 1000.0)
    st = summarize(recs, win, slo)
    done = cohort(recs, win)
    mine = {"slo_met": st["slo_met"], "completed": st["completed"], "cohort": st["cohort"],
            "ttft": [r.ttft for r in done if r.ttft is not None],
            "itl": [x for r in done for x in r.itls()],
            "out_tokens_in_window": sum(1 for r in recs for t in r.token_times if win[0] <= t <= win[1]),
            "idle_forwards": dp.idle_forwards, "iters": iters, "init_s": init_s,
            "status": 0 if a.cpu else K.scratch(device).read_status(),
            # this rank's engine steps over the whole run, by kind (decode /
            # mixed / prefill): what an iteration costs and what it carries
            "steps": rp.step_profile((0.0, float("inf")))}
    allr = [None] * world
    dist.all_gather_object(allr, mine, group=gloo)
    if rank == 0:
        ttft = [x for r in allr for x in r["ttft"]]
        itl = [x for r in allr for x in r["itl"]]
        out = {
            "metric": f"goodput req/s within TTFT / ITL p99 SLO on the {a.trace} trace; output tokens/s",
            "model": a.model, "parallelism": f"EP{world} + DP-attention{world}",
            "a2a": "nccl" if a.nccl_a2a else ("gloo" if a.cpu else "fused NVLink peer-store dispatch / return"),
            "rate": a.rate, "window_s": a.duration,
            "goodput_rps": round(sum(r["slo_met"] for r in allr) / a.duration, 4),
            "arrived": sum(r["cohort"] for r in allr), "completed": sum(r["completed"] for r in allr),
            "slo_met": sum(r["slo_met"] for r in allr),
            "slo": {"ttft_s": a.ttft_slo, "itl_p99_ms": a.itl_slo_ms},
            "output_tok_s": round(sum(r["out_tokens_in_window"] for r in allr) / a.duration, 1),
            "ttft_p50_s": round(percentile(ttft, 50), 3) if ttft else None,
            "ttft_p99_s": round(percentile(ttft, 99), 3) if ttft else None,
            "itl_p50_ms": round(1000 * percentile(itl, 50), 2) if itl else None,
            "itl_p99_ms": round(1000 * percentile(itl, 99), 2) if itl else None,
            "idle_forwards": [r["idle_forwards"] for r in allr], "iters": allr[0]["iters"],
            "init_s": round(max(r["init_s"] for r in allr), 1), "kernel_status": [r["status"] for r in allr],
            "step_profile_rank0": allr[0]["steps"],
            "data": "synthetic random tokens, random-init fp8 weights", "timing": "CUDA events per rank",
        }
        print(json.dumps(out), flush=True)
    dist.barrier(group=gloo)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

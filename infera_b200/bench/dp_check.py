"""Data-parallel attention + expert-parallel MoE engines against one
engine with all experts, on the DeepSeek-V3-shaped MLA model.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m infera_b200.bench.dp_check [--cpu] [--model tiny-moe] [--fused]

Every rank builds the same weights (one seed), keeps E / N experts, and
serves its own prompts (rank r gets prompts r, r + N, ...; ranks with fewer
prompts run idle forwards to stay in step). Each rank also runs a
single-process engine with the full expert set on its prompts and compares
the greedy outputs token by token. Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from infera_b200.engine.dp_attention import DPAttentionEngine, EPSpec
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--model", default="tiny-moe")
    ap.add_argument("--fused", action="store_true")
    ap.add_argument("--prompts", type=int, default=5)
    ap.add_argument("--max-tokens", type=int, default=6)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.cpu:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
        group = None
    else:
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        group = None
    gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    cfg = EngineConfig(model=a.model, use_cuda_graphs=False, num_pages=128, max_batched_tokens=64, max_num_seqs=4)
    g = torch.Generator().manual_seed(11)
    vocab = 1024 if a.cpu else 4096
    prompts = [torch.randint(0, vocab, (int(n),), generator=g).tolist()
               for n in torch.randint(3, 60, (a.prompts,), generator=g)]
    mine = prompts[rank::world]
    dp = DPAttentionEngine(cfg, EPSpec(rank, world, group=group, gloo=gloo, fused=a.fused and not a.cpu), device=dev)
    # odd ranks stop earlier so they run idle forwards while the others finish
    n_out = a.max_tokens if rank % 2 == 0 else max(1, a.max_tokens // 3)
    sp = SamplingParams(max_tokens=n_out, ignore_eos=True)
    for i, p in enumerate(mine):
        dp.add_request(f"r{rank}-{i}", p, sp)
    got = dp.run_until_idle()
    outs = [got.get(f"r{rank}-{i}", []) for i in range(len(mine))]
    # the same prompts through one engine holding every expert
    ref = LLMEngine(cfg, device=dev).generate(mine, sp) if mine else []
    agree = sum(int(x == y) for o, r in zip(outs, ref) for x, y in zip(o, r))
    total = sum(len(r) for r in ref)
    res = {"rank": rank, "prompts": len(mine), "tokens": total, "agree": agree,
           "idle_forwards": dp.idle_forwards, "complete": all(len(o) == n_out for o in outs)}
    allr = [None] * world
    dist.all_gather_object(allr, res, group=gloo)
    if rank == 0:
        print(json.dumps({"world": world, "ranks": allr,
                          "agreement": sum(r["agree"] for r in allr) / max(1, sum(r["tokens"] for r in allr))}),
              flush=True)
    for lw in dp.engine.model.w.layers:
        if "moe" in lw and hasattr(lw["moe"], "close"):
            lw["moe"].close()
    dist.barrier(group=gloo)
    dist.destroy_process_group()
    if not all(r["complete"] for r in allr):
        raise SystemExit("a rank did not finish its requests")


if __name__ == "__main__":
    main()

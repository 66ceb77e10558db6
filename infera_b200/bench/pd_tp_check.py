"""Prefill/decode pair of tensor-parallel instances.

    python -m torch.distributed.run --nproc-per-node W --master-addr 127.0.0.1 \\
        -m infera_b200.bench.pd_tp_check [--cpu] [--model tiny-dense]

Each process holds rank r of three tensor-parallel groups of width W: a
mixed instance (the oracle), a prefill instance and a decode instance (on
GPU all three on ``cuda:r``; the push from prefill rank r into decode rank r
is then a local copy, the protocol is the one a pair on separate GPUs runs).
Rank 0 leads every group; the others mirror its steps. Two requests go
through the pair: one whose prompt takes several chunks (its pages are
pushed layer by layer inside the last chunk's forward) and one pushed after
its prompt. Every prefill rank pushes its own KV-head shard into the same
rank of the decode group; the decode group computes only each prompt's
last token. Rank 0 prints one JSON line: the decode outputs against the
mixed instance's, and per-rank push counters.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.engine.tp_engine import TPLeader, follower_loop, follower_step
from infera_b200.parallel.comm import TPComm


def _group_pair(cpu: bool):
    coll = dist.new_group(backend="gloo" if cpu else "nccl", timeout=timedelta(seconds=120))
    ctrl = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    return coll, ctrl


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-dense")
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--tokens", type=int, default=5)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if a.cpu:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    else:
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from infera_b200.models.config import get_config

    hidden = get_config(a.model).hidden
    tps = {}
    for name in ("mix", "pre", "dec"):
        coll, ctrl = _group_pair(a.cpu)
        tps[name] = TPComm(rank, world, dev, hidden, nccl_group=coll, gloo_group=ctrl, max_rows=256)

    def eng(name, **kw):
        cfg = EngineConfig(model=a.model, use_cuda_graphs=False, num_pages=256, max_num_seqs=8, **kw)
        return LLMEngine(cfg, device=dev, tp=tps[name])

    mix = eng("mix", max_batched_tokens=256)
    pre = eng("pre", max_batched_tokens=32, disagg_mode="prefill")
    dec = eng("dec", max_batched_tokens=256, disagg_mode="decode", kv_push_endpoint="local://pd-tp-check")
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(10, 1000, (n,), generator=g).tolist() for n in (90, 20)]
    sp = SamplingParams(max_tokens=a.tokens, ignore_eos=True)

    # the oracle: the mixed tensor-parallel instance
    if rank == 0:
        lead = TPLeader(mix, tps["mix"].gloo)
        ref = lead.generate(prompts, sp)
        lead.shutdown()
    else:
        follower_loop(mix, tps["mix"].gloo)

    outs: dict[str, list[int]] = {}
    if rank == 0:
        pl, dl = TPLeader(pre, tps["pre"].gloo), TPLeader(dec, tps["dec"].gloo)
        ep = dec.pd_rendezvous.endpoint
        for i, p in enumerate(prompts):
            room = 100 + i
            dec.add_request(f"d{i}", p, SamplingParams(max_tokens=a.tokens, ignore_eos=True,
                                                       kv_transfer={"do_remote_prefill": True, "room": room}))
            outs[f"d{i}"] = []
        dl.step()   # parks both requests and publishes their pages
        for i, p in enumerate(prompts):
            pre.add_request(f"p{i}", p, SamplingParams(max_tokens=1, ignore_eos=True, kv_transfer={
                "do_remote_decode": True, "room": 100 + i, "decode_kv_endpoint": ep, "layerwise": i == 0}))
        t0 = time.monotonic()
        while pre.has_unfinished() or dec.has_unfinished():
            if time.monotonic() - t0 > 60:
                break
            pl.step()
            for o in dl.step():
                outs[o.request_id].extend(o.new_token_ids)
            time.sleep(0.005)   # lets the agent thread resolve page lists between chunks
        pl.shutdown()
        dl.shutdown()
    else:
        follower_step(dec, tps["dec"].gloo)
        while True:
            a_ = follower_step(pre, tps["pre"].gloo)
            b_ = follower_step(dec, tps["dec"].gloo)
            if not a_ and not b_:
                break
    st = {"rank": rank, "pushes": pre.pd_agent.stats["pushes"] if pre.pd_agent else 0,
          "layerwise": pre.pd_agent.stats["layerwise"] if pre.pd_agent else 0,
          "pages": pre.pd_agent.stats["pages"] if pre.pd_agent else 0,
          "decode_prompt_tokens": dec.counters["prompt_tokens"], "unfinished": dec.has_unfinished()}
    allst = [None] * world
    dist.all_gather_object(allst, st, group=tps["mix"].gloo)
    if rank == 0:
        got = [outs[f"d{i}"] for i in range(len(prompts))]
        print(json.dumps({"tp": world, "model": a.model, "equal_to_mixed": got == ref, "outputs": got,
                          "reference": ref, "ranks": allst}), flush=True)
    for e in (mix, pre, dec):
        e.close()
    for t in tps.values():
        t.close()
    dist.barrier(group=tps["mix"].gloo)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Tensor-parallel engine against the single-GPU engine, and its decode
step time with the fused NVLink all-reduce vs NCCL.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m infera_b200.bench.tp_engine_check [--model llama-3.1-8b] [--batch 32]

Rank 0 leads (TPLeader), the others follow. Prints JSON lines on rank 0:
the greedy-token agreement and last-logits error against a TP=1 engine
built on rank 0's GPU, then the mean device time of decode-only steps
(CUDA events around each leader step, warm-up first).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.engine.tp_engine import TPLeader, follower_loop
from infera_b200.parallel.launch import init_tp


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--decode-steps", type=int, default=64)
    ap.add_argument("--no-reference", action="store_true")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp, rank, dev = init_tp(world, model=a.model)
    cfg = EngineConfig(model=a.model, max_num_seqs=max(64, a.batch), max_batched_tokens=4096, num_pages=4096)
    eng = LLMEngine(cfg, device=dev, tp=tp)
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(1000, 60000, (a.prompt_len,), generator=g).tolist() for _ in range(a.batch)]
    sp = SamplingParams(max_tokens=a.decode_steps, ignore_eos=True)
    if rank > 0:
        follower_loop(eng, tp.gloo)
        follower_loop(eng, tp.gloo)
        eng.close()
        tp.close()
        dist.destroy_process_group()
        return
    lead = TPLeader(eng, tp.gloo)
    # correctness run (records the last-step logits of request 0)
    outs = lead.generate(prompts[:4], SamplingParams(max_tokens=8, ignore_eos=True))
    lead.shutdown()
    res = {"model": a.model, "tp": world, "fused": tp.fused}
    if not a.no_reference:
        ref_eng = LLMEngine(EngineConfig(model=a.model, max_num_seqs=64, max_batched_tokens=4096, num_pages=4096),
                            device=dev)
        ref = ref_eng.generate(prompts[:4], SamplingParams(max_tokens=8, ignore_eos=True))
        agree = sum(x == y for o, r in zip(outs, ref) for x, y in zip(o, r)) / sum(len(r) for r in ref)
        res["greedy_agreement"] = round(agree, 4)
        # random-init weights put many next tokens within rounding distance of
        # each other: at each sequence's first divergence, how far below the
        # single-GPU model's best logit the tensor-parallel choice is,
        # relative to the largest logit magnitude (near 0: a rounding tie)
        worst, div = 0.0, 0
        for p, o, r in zip(prompts[:4], outs, ref):
            i = next((j for j, (x, y) in enumerate(zip(o, r)) if x != y), None)
            if i is None:
                continue
            div += 1
            ref_eng.generate([p + o[:i]], SamplingParams(max_tokens=1, ignore_eos=True))
            lg = ref_eng.runner.last_logits[-1].float()
            worst = max(worst, float(lg.max() - lg[o[i]]) / float(lg.abs().max()))
        res["divergences"] = div
        res["max_rel_gap_at_divergence"] = round(worst, 5)
        ref_eng.close()
        del ref_eng
        torch.cuda.empty_cache()
    # decode step time: prefill the batch, then time decode-only steps
    lead2 = TPLeader(eng, tp.gloo)
    for i, p in enumerate(prompts):
        eng.add_request(f"t{i}", p, sp)
    while eng.scheduler.waiting or any(r.num_computed < len(r.prompt_token_ids) for r in eng.scheduler.running):
        lead2.step()
    times = []
    for _ in range(min(a.decode_steps - 8, 48)):
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        lead2.step()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    while eng.has_unfinished():
        lead2.step()
    lead2.shutdown()
    t = times[8:]
    res.update({"batch": a.batch, "context": a.prompt_len, "decode_ms_per_step": round(sum(t) / len(t), 3),
                "status": int(__import__("infera_b200.ops.kernels", fromlist=["x"]).scratch(dev).read_status())})
    print(json.dumps(res), flush=True)
    eng.close()
    tp.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

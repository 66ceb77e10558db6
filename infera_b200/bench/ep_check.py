"""Expert-parallel MoE layer against the single-device layer, and its
device time (one rank per device, or gloo processes on CPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m infera_b200.bench.ep_check [--cpu] [--tokens 64] [--hidden 7168 --ffn 2048 --experts 256]

Every rank builds the same full layer from one seed, keeps its expert
shard, routes its own slice of the tokens, and compares its output rows
with the full layer applied to the same tokens on one device.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from infera_b200.models.moe import MoELayer
from infera_b200.parallel.ep import EPMoE


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--tokens", type=int, default=64, help="tokens per rank")
    ap.add_argument("--hidden", type=int, default=1024)
    ap.add_argument("--ffn", type=int, default=512)
    ap.add_argument("--experts", type=int, default=32)
    ap.add_argument("--top-k", type=int, default=4)
    ap.add_argument("--iters", type=int, default=0)
    ap.add_argument("--fused", action="store_true", help="NVLink peer-store dispatch / return (GPUs)")
    ap.add_argument("--fp8", action="store_true", help="e4m3 experts with 128x128 block scales")
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.cpu:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    else:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=120)) if not a.cpu else None
    full = MoELayer(a.hidden, a.ffn, a.experts, a.top_k, n_groups=4, topk_groups=2, routed_scaling=2.0,
                    num_shared=1, device="cpu", seed=7, weight_dtype="fp8" if a.fp8 else "bf16")
    g = torch.Generator().manual_seed(11)
    x_all = torch.randn(world * a.tokens, a.hidden, generator=g).to(torch.bfloat16)
    x = x_all[rank * a.tokens:(rank + 1) * a.tokens].contiguous()
    ids, wts = full.route(x)  # same routing on both paths
    ref = full.forward(x, ids, wts)
    ep = EPMoE(full, rank, world, device=dev, fused=a.fused, max_tokens=a.tokens, gloo_group=gloo)
    y = ep.forward(x.to(dev), ids.to(dev), wts.to(dev))
    if dev.type == "cuda":
        torch.cuda.synchronize()
    err = float((y.float().cpu() - ref.float()).norm() / ref.float().norm())
    res = {"rank": rank, "world": world, "fused": ep.fused, "rel_err": round(err, 5),
           "sent_rows": ep.stats["sent_rows"], "recv_rows": ep.stats["recv_rows"]}
    if dev.type == "cuda":
        from infera_b200.ops import kernels as K

        res["status"] = K.scratch(dev).read_status()
    if a.iters and dev.type == "cuda":
        xd, idd, wd = x.to(dev), ids.to(dev), wts.to(dev)
        for _ in range(3):
            ep.forward(xd, idd, wd)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for _ in range(a.iters):
            ep.forward(xd, idd, wd)
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res["ms_per_layer"] = round(float(t.item()), 4)
    out = [None] * world
    dist.all_gather_object(out, res)
    if rank == 0:
        print(json.dumps({"ranks": out, "max_rel_err": max(r["rel_err"] for r in out)}), flush=True)
    dist.barrier()
    if hasattr(ep, "close"):
        ep.close()
    dist.destroy_process_group()
    if err > 2e-2:
        raise SystemExit(f"expert-parallel mismatch on rank {rank}: {err}")


if __name__ == "__main__":
    main()

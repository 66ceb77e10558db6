"""Row-parallel GEMM + all-reduce + residual add + RMSNorm across a
tensor-parallel group: the fused NVLink path against the NCCL baseline.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m infera_b200.bench.tp_comm_bench [--rows 64] [--hidden 8192] [--k-total 8192]

Each rank holds a K-slice of the weight (``k_total / N`` columns) and of the
activations; the full product is the sum over ranks. Checks both paths
against a single-GPU fp32 computation of the whole problem, then times
each (CUDA events on the launching stream, warm-up first, max over ranks)
and prints one JSON line per row count on rank 0. The roofline for the
fused path is the slower of the GEMM's FLOPs at the measured bf16 peak and
the bytes each rank must push over NVLink at 770 GB/s and the weight
bytes at the measured HBM copy bandwidth (small row counts are
weight-bandwidth bound). Timed loops are captured in CUDA graphs.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from infera_b200.ops import kernels as K
from infera_b200.parallel.comm import TPComm

# roofline denominators measured on B200: copy bandwidth (read + write bytes),
# bf16 GEMM burst rate, NVLink peer-copy rate per direction
PEAK_HBM = 6418.2e9
PEAK_BF16 = 1675.3e12
PEAK_PEER = 770e9


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", default="1,16,64,128,256")
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--k-total", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--check-only", action="store_true")
    ap.add_argument("--lm-head", type=int, default=0, metavar="VOCAB",
                    help="instead: the vocab-parallel LM head (each rank owns VOCAB / N rows of the weight) with "
                         "the all-gather of the logits fused into its GEMM, against GEMM + NCCL all-gather")
    ap.add_argument("--one-shot-rows", type=int, default=0,
                    help="largest row count for the one-shot path; larger rows take the two-shot "
                         "(reduce-scatter + all-gather) path (0: one-shot for every row count)")
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    nccl = gloo = None
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        nccl = dist.group.WORLD
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    H, KT = a.hidden, a.k_total
    Ks = KT // world
    rows = [int(r) for r in a.rows.split(",")]
    if a.lm_head:
        return _lm_head(a, rank, world, dev, nccl, gloo, rows)
    if a.one_shot_rows:
        comm = TPComm(rank, world, dev, H, max_rows=a.one_shot_rows, nccl_group=nccl, gloo_group=gloo,
                      max_rows_rs=max(rows), two_shot=True)
    else:
        comm = TPComm(rank, world, dev, H, max_rows=max(rows), nccl_group=nccl, gloo_group=gloo)
    g = torch.Generator(device=dev).manual_seed(1234)  # same full tensors on every rank
    worst = 0.0
    results = []
    for M in rows:
        x_full = (torch.randn(M, KT, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        w_full = (torch.randn(H, KT, device=dev, generator=g) / KT ** 0.5).to(torch.bfloat16)
        h0 = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
        nw = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).to(torch.bfloat16)
        xs = x_full[:, rank * Ks:(rank + 1) * Ks].contiguous()
        ws = w_full[:, rank * Ks:(rank + 1) * Ks].contiguous()
        ref_h = (h0.float() + x_full.float() @ w_full.float().t()).to(torch.bfloat16)
        ref_x = (ref_h.float() * torch.rsqrt(ref_h.float().pow(2).mean(-1, keepdim=True) + 1e-5) * nw.float())
        out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        for parity in (0, 1, 0, 1):  # alternate like the layers do
            h = h0.clone()
            comm.gemm_allreduce_add_rmsnorm(xs, ws, h, nw, 1e-5, out, parity)
        torch.cuda.synchronize()
        err = float((out.float() - ref_x).norm() / ref_x.norm())
        two = comm.uses_two_shot(M)
        if two:  # the residual is kept by each row block's owner only
            own = (torch.arange(M, device=dev) // 128) % world == rank
            herr = float((h[own].float() - ref_h[own].float()).norm() / ref_h[own].float().norm()) if own.any() else 0.0
        else:
            herr = float((h.float() - ref_h.float()).norm() / ref_h.float().norm())
        # NCCL baseline on the same problem
        base = TPComm(rank, world, dev, H, max_rows=max(rows), nccl_group=nccl, gloo_group=gloo, fused=False)
        hb = h0.clone()
        outb = torch.empty_like(out)
        base.gemm_allreduce_add_rmsnorm(xs, ws, hb, nw, 1e-5, outb, 0)
        torch.cuda.synchronize()
        errb = float((outb.float() - ref_x).norm() / ref_x.norm())
        status = K.scratch(dev).read_status()
        worst = max(worst, err, errb)
        res = {"rows": M, "hidden": H, "k_per_rank": Ks, "world": world, "path": "two-shot" if two else "one-shot",
               "rel_err_fused": err, "rel_err_residual": herr, "rel_err_nccl": errb, "status": status}
        if not a.check_only:
            # rotate weight copies totalling > 256 MB so every launch reads HBM, not L2
            nrep = max(1, -(-(256 << 20) // (H * Ks * 2)))
            wl = [ws] + [ws.clone() for _ in range(nrep - 1)]
            for name, c in (("fused", comm), ("nccl", base)):
                hh = h0.clone()
                for i in range(4):
                    c.gemm_allreduce_add_rmsnorm(xs, ws, hh, nw, 1e-5, out, i & 1)
                torch.cuda.synchronize()
                if name == "fused" and two:
                    # host-counted rounds: timed eagerly (large row counts, launch cost negligible)
                    if world > 1:
                        dist.barrier(group=gloo)
                    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
                    s.record()
                    for i in range(a.iters):
                        c.gemm_allreduce_add_rmsnorm(xs, wl[i % nrep], hh, nw, 1e-5, out, i & 1)
                    e.record()
                    torch.cuda.synchronize()
                    t = torch.tensor([s.elapsed_time(e) * 1000 / a.iters], device=dev)
                    if world > 1:
                        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=nccl)
                    res[f"us_{name}"] = round(float(t.item()), 2)
                    continue
                # capture the loop in a CUDA graph: device time, not the
                # host's launch rate
                gr = torch.cuda.CUDAGraph()
                st = torch.cuda.Stream()
                st.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(st):
                    with torch.cuda.graph(gr, stream=st):
                        for i in range(a.iters):
                            c.gemm_allreduce_add_rmsnorm(xs, wl[i % nrep], hh, nw, 1e-5, out, i & 1)
                torch.cuda.current_stream().wait_stream(st)
                torch.cuda.synchronize()
                gr.replay()  # warm
                torch.cuda.synchronize()
                if world > 1:
                    dist.barrier(group=gloo)
                s, e = torch.cuda.Event(True), torch.cuda.Event(True)
                s.record()
                gr.replay()
                e.record()
                torch.cuda.synchronize()
                us = s.elapsed_time(e) * 1000 / a.iters
                del gr
                t = torch.tensor([us], device=dev)
                if world > 1:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=nccl)
                res[f"us_{name}"] = round(float(t.item()), 2)
            flops = 2.0 * M * H * Ks
            w_bytes = H * Ks * 2
            push_bytes = (2 * (world - 1) / world if two else (world - 1)) * M * H * 2
            res["roofline_us"] = round(max(flops / PEAK_BF16, w_bytes / PEAK_HBM, push_bytes / PEAK_PEER) * 1e6, 2)
            res["roofline_note"] = (f"max(FLOPs / {PEAK_BF16 / 1e12:.1f} TF, weight bytes / {PEAK_HBM / 1e9:.1f} GB/s, "
                                    f"pushed bytes / {PEAK_PEER / 1e9:.0f} GB/s)")
            res["frac_fused"] = round(res["roofline_us"] / res["us_fused"], 3)
        results.append(res)
        if rank == 0:
            print(json.dumps(res), flush=True)
    comm.close()
    if world > 1:
        dist.barrier(group=gloo)
        dist.destroy_process_group()
    if worst > 2e-2:
        raise SystemExit(f"tensor-parallel all-reduce mismatch: worst relative error {worst}")


def _graph_time(fn, iters: int, world: int, gloo, nccl, dev) -> float:
    """Device microseconds per call of ``fn`` replayed from a CUDA graph, max
    over ranks."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(gr, stream=st):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream().wait_stream(st)
    gr.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group=gloo)
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    gr.replay()
    e.record()
    torch.cuda.synchronize()
    del gr
    t = torch.tensor([s.elapsed_time(e) * 1000 / iters], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=nccl)
    return float(t.item())


def _lm_head(a, rank, world, dev, nccl, gloo, rows) -> None:
    """Vocab-parallel LM head: logits = x @ W.T with W split by rows over the
    ranks; every rank needs every column of the logits."""
    H, V = a.hidden, a.lm_head
    n = V // world
    comm = TPComm(rank, world, dev, H, max_rows=8, nccl_group=nccl, gloo_group=gloo)
    comm.ensure_gather(max(rows), V)
    base = TPComm(rank, world, dev, H, max_rows=8, nccl_group=nccl, gloo_group=gloo, fused=False)
    g = torch.Generator(device=dev).manual_seed(99)
    w_full = (torch.randn(V, H, device=dev, generator=g) / H ** 0.5).to(torch.bfloat16)
    w_loc = w_full[rank * n:(rank + 1) * n].contiguous()
    worst = 0.0
    for M in rows:
        x = (torch.randn(M, H, device=dev, generator=g)).to(torch.bfloat16)
        ref = x.float() @ w_full.float().t()
        got = comm.gemm_allgather_cols(x, w_loc).clone()
        torch.cuda.synchronize()
        err = float((got.float() - ref).norm() / ref.norm())
        errb = float((base.all_gather_cols(K.linear(x, w_loc)).float() - ref).norm() / ref.norm())
        worst = max(worst, err, errb)
        res = {"case": "lm_head", "rows": M, "hidden": H, "vocab": V, "world": world, "rel_err_fused": err,
               "rel_err_nccl": errb, "status": K.scratch(dev).read_status(),
               "fused": comm.uses_fused_gather(M, n, w_loc)}
        if not a.check_only:
            nrep = max(1, -(-(256 << 20) // (n * H * 2)))
            wl = [w_loc] + [w_loc.clone() for _ in range(nrep - 1)]
            it = [0]

            def fused():
                it[0] += 1
                comm.gemm_allgather_cols(x, wl[it[0] % nrep])

            def nccl_path():
                it[0] += 1
                base.all_gather_cols(K.linear(x, wl[it[0] % nrep]))

            res["us_fused"] = round(_graph_time(fused, a.iters, world, gloo, nccl, dev), 2)
            res["us_nccl"] = round(_graph_time(nccl_path, a.iters, world, gloo, nccl, dev), 2)
            w_bytes = n * H * 2
            push = (world - 1) * M * n * 2
            res["roofline_us"] = round(max(2.0 * M * n * H / PEAK_BF16, w_bytes / PEAK_HBM, push / PEAK_PEER) * 1e6, 2)
            res["frac_fused"] = round(res["roofline_us"] / res["us_fused"], 3)
        if rank == 0:
            print(json.dumps(res), flush=True)
    comm.close()
    if world > 1:
        dist.barrier(group=gloo)
        dist.destroy_process_group()
    if worst > 2e-2:
        raise SystemExit(f"LM-head gather mismatch: worst relative error {worst}")


if __name__ == "__main__":
    main()

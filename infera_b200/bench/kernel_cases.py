"""Standalone kernel cases for timing and profiling (small device
footprint, inputs larger than L2 where the case is memory-bound).

    python -m infera_b200.bench.kernel_cases <case> [<case> ...] [--iters N]

Cases: gemm_prefill (2048x6144x4096 bf16), gemm_decode (64 tokens x
28672x4096, SwiGLU epilogue), gemm_lmhead (64x128256x4096), decode_attn
(32 seqs x 8192 keys, GQA 32/8), decode_attn_shared / decode_attn_private
(24 seqs, 4096-token prefix shared by groups of 12 or all pages private, +1k-12k
tail each), fp8_decode (64 x 28672 x 8192 e4m3,
block scales, SwiGLU), fp8_prefill (4096 x 8192 x 8192 e4m3), mla_decode (64
queries x 128 heads over 4096 latent keys each), prefill_attn (2048 queries over 2048 keys,
causal), prefill_attn_prefix (1024 queries over 8192 keys), prefill_attn_chunk
(a 224-token chunk over 8192 cached keys: key shares), mla_prefill /
mla_prefill_prefix (DeepSeek-V3 MLA prompt chunk, 128 heads: 2048 queries
over 2048 keys causal, or 1024 over 8192; the non-absorbed path against the
absorbed latent kernel on the same queries). Prints one JSON
line per case: mean CUDA-event time per launch after 3 warm-up launches, and the
achieved TFLOP/s or GB/s.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from infera_b200.ops import kernels as K


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def run_case(case: str, iters: int) -> dict:
    dev = "cuda"
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    if case.startswith("gemm"):
        M, N, Kd, swiglu = {"gemm_prefill": (2048, 6144, 4096, False), "gemm_decode": (64, 28672, 4096, True),
                            "gemm_lmhead": (64, 128256, 4096, False),
                            # a mixed step: ~60 decodes + a 224-token prompt chunk
                            "gemm_mixed": (288, 28672, 4096, True),
                            "gemm_mixed_down": (288, 4096, 14336, False)}[case]
        x = torch.randn(M, Kd, device=dev, generator=g).to(bf)
        w = (torch.randn(N, Kd, device=dev, generator=g) / math.sqrt(Kd)).to(bf)
        ms = _time(lambda: K.linear(x, w, swiglu=swiglu), iters)
        fl = 2 * M * N * Kd
        by = (M * Kd + N * Kd + M * (N // 2 if swiglu else N)) * 2
        return {"case": case, "ms": ms, "tflops": fl / ms / 1e9, "gbs": by / ms / 1e6, "plan": K.gemm_plan(M, N, Kd)}
    if case.startswith("fp8_"):
        from infera_b200.ops import fp8

        M, N, Kd, swiglu = {"fp8_decode": (64, 28672, 8192, True), "fp8_prefill": (4096, 8192, 8192, False),
                            "fp8_decode_small": (8, 10240, 8192, False),
                            "fp8_prefill_small": (2048, 4096, 4096, False)}[case]
        x = torch.randn(M, Kd, device=dev, generator=g).to(bf)
        wq = fp8.quantize_weight(torch.randn(N, Kd, device=dev, generator=g) / math.sqrt(Kd))
        q, sf = fp8.quant_act(x)
        ms = _time(lambda: fp8.gemm_fp8(q, sf, wq, swiglu=swiglu), iters)
        ms_q = _time(lambda: fp8.linear(x, wq, swiglu=swiglu), iters)
        fl = 2 * M * N * Kd
        by = M * Kd + N * Kd + N * Kd // 16384 + M * (N // 2 if swiglu else N) * 2
        return {"case": case, "ms": ms, "ms_with_act_quant": ms_q, "tflops": fl / ms / 1e9, "gbs": by / ms / 1e6}
    if case in ("mla_decode", "mla_decode_small", "mla_decode_contig"):
        # _contig: each sequence's pages consecutive (as the page allocator
        # hands out prompt pages), the others placed at random
        from infera_b200.ops import mla as M

        B, L, hq = (16, 4096, 128) if case == "mla_decode_small" else (64, 4096, 128)
        pages = B * L // 16
        cache = torch.randn(pages * 16, 576, device=dev, generator=g).to(bf)
        if case == "mla_decode_contig":
            bt = torch.arange(pages, device=dev, dtype=torch.int32).view(B, -1)
        else:
            bt = torch.randperm(pages, device=dev, dtype=torch.int32).view(B, -1)
        q = (torch.randn(B, hq, 576, device=dev, generator=g) * 0.05).to(bf)
        rows = torch.arange(B, dtype=torch.int32, device=dev)
        kvl = torch.full((B,), L, dtype=torch.int32, device=dev)
        ms = _time(lambda: M.mla_attention(q, cache, bt, rows, kvl, 0.07, max_kvlen=L), iters)
        fl = 2 * B * hq * L * (576 + 512)            # useful FLOPs (S and PV once)
        by = B * L * 576 * 2 + B * hq * (576 + 512) * 2
        return {"case": case, "ms": ms, "tflops": fl / ms / 1e9, "gbs": by / ms / 1e6,
                "splits": M.mla_splits(B, L, K._num_sms())}
    hq, hkv, D = 32, 8, 128
    if case in ("decode_attn", "decode_attn_contig", "decode_attn_48x2048", "decode_attn_48x2048_contig"):
        # decode_attn: every page placed at random; _contig: each sequence's
        # pages consecutive (eight-page runs load as one box per half);
        # 48x2048: the serving bench's decode batch shape
        B, L = (48, 2048) if "48x2048" in case else (32, 8192)
        pages = B * L // 16
        kc = torch.randn(pages * 16, hkv * D, device=dev, generator=g).to(bf)
        vc = torch.randn(pages * 16, hkv * D, device=dev, generator=g).to(bf)
        if not case.endswith("contig"):
            bt = torch.randperm(pages, device=dev, dtype=torch.int32).view(B, -1)
        else:
            bt = torch.arange(pages, device=dev, dtype=torch.int32).view(B, -1)
        sl = torch.full((B,), L, dtype=torch.int32, device=dev)
        q = torch.randn(B, hq * D, device=dev, generator=g).to(bf)
        sp = K.decode_splits(B, hkv, L)
        ms = _time(lambda: K.attn_decode(q, kc, vc, bt, sl, hq, hkv, 1 / math.sqrt(D), splits=sp), iters)
        by = 2 * B * L * hkv * D * 2
        return {"case": case, "ms": ms, "gbs": by / ms / 1e6, "splits": sp}
    if case in ("decode_attn_shared", "decode_attn_private"):
        # the serving trace's decode batch: 24 sequences in 2 groups of 12 that
        # share a 4096-token system prefix (the same physical pages, as the
        # prefix cache hands them out), then private tails of 1k-12k tokens;
        # "private": the same lengths with every page distinct
        B, P = 24, 4096
        gg = torch.Generator().manual_seed(1)
        tails = torch.randint(1000, 12000, (B,), generator=gg).tolist()
        lens = [P + t for t in tails]
        shared = case == "decode_attn_shared"
        n_pages = (2 * P // 16 if shared else 0) + sum(((n if not shared else n - P) + 15) // 16 for n in lens)
        kc = torch.randn(n_pages * 16, hkv * D, device=dev, generator=g).to(bf)
        vc = torch.randn(n_pages * 16, hkv * D, device=dev, generator=g).to(bf)
        perm = torch.randperm(n_pages, generator=gg).tolist()
        width = max((n + 15) // 16 for n in lens)
        bt = torch.zeros(B, width, dtype=torch.int32)
        nxt = 2 * P // 16 if shared else 0
        for b, n in enumerate(lens):
            row = []
            if shared:
                grp = b % 2
                row += perm[grp * (P // 16):(grp + 1) * (P // 16)]
            need = (n + 15) // 16 - len(row)
            row += perm[nxt:nxt + need]
            nxt += need
            bt[b, :len(row)] = torch.tensor(row, dtype=torch.int32)
        bt = bt.to(dev)
        sl = torch.tensor(lens, dtype=torch.int32, device=dev)
        q = torch.randn(B, hq * D, device=dev, generator=g).to(bf)
        import os

        tps = int(os.environ.get("INFERA_DECODE_TPS", "0"))       # tiles per split (0: even split)
        l2 = int(os.environ.get("INFERA_DECODE_L2", "0"))
        sp = K.decode_splits(B, hkv, max(lens)) if tps == 0 else -(-max(lens) // (tps * 128))
        ms = _time(lambda: K.attn_decode(q, kc, vc, bt, sl, hq, hkv, 1 / math.sqrt(D), splits=sp,
                                         tiles_per_split=tps, l2_policy=l2), iters)
        ref = K.attn_decode(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), hq, hkv, 1 / math.sqrt(D)).float()
        got = K.attn_decode(q, kc, vc, bt, sl, hq, hkv, 1 / math.sqrt(D), splits=sp, tiles_per_split=tps,
                            l2_policy=l2).float().cpu()
        by_all = sum(lens) * hkv * D * 2 * 2
        by_unique = n_pages * 16 * hkv * D * 2 * 2
        return {"case": case, "ms": ms, "gbs_all_keys": by_all / ms / 1e6, "gbs_unique_pages": by_unique / ms / 1e6,
                "bytes_all": by_all, "bytes_unique": by_unique, "splits": sp, "tiles_per_split": tps,
                "l2_policy": l2, "rel_err": float((got - ref).norm() / ref.norm())}
    if case in ("prefill_attn", "prefill_attn_prefix", "prefill_attn_chunk", "prefill_attn_8k",
                "prefill_attn_32k"):
        ql, ctx = {"prefill_attn": (2048, 2048), "prefill_attn_prefix": (1024, 8192),
                   "prefill_attn_chunk": (224, 8192), "prefill_attn_8k": (8192, 8192),
                   "prefill_attn_32k": (8192, 32768)}[case]
        pages = ctx // 16
        kc = torch.randn(pages * 16, hkv * D, device=dev, generator=g).to(bf)
        vc = torch.randn(pages * 16, hkv * D, device=dev, generator=g).to(bf)
        bt = torch.arange(pages, device=dev, dtype=torch.int32).view(1, -1)
        q = torch.randn(ql, hq * D, device=dev, generator=g).to(bf)
        tiles = torch.tensor(K.prefill_tiles([ql]), dtype=torch.int32, device=dev)
        meta = [torch.tensor([v], dtype=torch.int32, device=dev) for v in (0, ql, ctx)]
        splits = K.prefill_kv_splits(hq, tiles.shape[0], ctx)
        ms = _time(lambda: K.attn_prefill(q, kc, vc, bt, *meta, tiles, hq, hkv, 1 / math.sqrt(D),
                                          kv_splits=splits), iters)
        keys = sum(ctx - ql + i + 1 for i in range(ql))
        res = {"case": case, "ms": ms, "tflops": 4 * keys * D * hq / ms / 1e9, "kv_splits": splits}
        if splits > 1:
            ms1 = _time(lambda: K.attn_prefill(q, kc, vc, bt, *meta, tiles, hq, hkv, 1 / math.sqrt(D),
                                               kv_splits=1), iters)
            res.update(ms_unsplit=ms1, speedup_vs_unsplit=ms1 / ms)
        if case == "prefill_attn_chunk":
            res["ms_by_splits"] = {sp: _time(lambda: K.attn_prefill(q, kc, vc, bt, *meta, tiles, hq, hkv,
                                                                    1 / math.sqrt(D), kv_splits=sp), iters)
                                   for sp in (1, 2, 4, 8)}
        # one 128-row query tile per CTA, for comparison
        t1 = torch.tensor(K.prefill_tiles([ql], 128), dtype=torch.int32, device=dev)
        s1 = K.prefill_kv_splits(hq, t1.shape[0], ctx)
        ref = K.attn_prefill(q, kc, vc, bt, *meta, t1, hq, hkv, 1 / math.sqrt(D), kv_splits=s1, tile_rows=128)
        got = K.attn_prefill(q, kc, vc, bt, *meta, tiles, hq, hkv, 1 / math.sqrt(D), kv_splits=splits)
        ms128 = _time(lambda: K.attn_prefill(q, kc, vc, bt, *meta, t1, hq, hkv, 1 / math.sqrt(D), kv_splits=s1,
                                             tile_rows=128), iters)
        res.update(tile_rows=K.PREFILL_TILE_ROWS, ms_tile128=ms128, tflops_tile128=4 * keys * D * hq / ms128 / 1e9,
                   max_abs_diff_vs_tile128=float((got.float() - ref.float()).abs().max()))
        return res
    if case in ("mla_prefill", "mla_prefill_prefix"):
        from infera_b200.ops import mla as M

        ql, ctx = (2048, 2048) if case == "mla_prefill" else (1024, 8192)
        hq = 128
        pages = ctx // 16
        cache = (torch.randn(pages * 16, 576, device=dev, generator=g) * 0.5).to(bf)
        bt = torch.arange(pages, device=dev, dtype=torch.int32).view(1, -1)
        qb = (torch.randn(ql, hq * 192, device=dev, generator=g) * 0.5).to(bf)
        q_full = (torch.randn(ql, hq, 576, device=dev, generator=g) * 0.5).to(bf)
        w_uk = (torch.randn(hq, 512, 128, device=dev, generator=g) / math.sqrt(512)).to(bf)
        w_uv = (torch.randn(hq, 128, 512, device=dev, generator=g) / math.sqrt(512)).to(bf)
        w_up = M.kv_up_weight(w_uk, w_uv)
        tiles = torch.tensor(K.prefill_tiles([ql], 128), dtype=torch.int32, device=dev)
        meta = [torch.tensor([v], dtype=torch.int32, device=dev) for v in (0, ql, ctx)]
        scale = M.default_scale(128, 64)
        run = lambda: M.mla_prefill(qb, q_full, cache, bt, None, ([ql], [ctx]), *meta, tiles, w_up, hq, 128,  # noqa
                                    128, scale)
        ms = _time(run, iters)
        keys = sum(ctx - ql + i + 1 for i in range(ql))
        attn_fl = 2 * keys * hq * (192 + 128)
        up_fl = 2 * ctx * 512 * hq * 256
        # the absorbed latent kernel on the same queries (one per token)
        rows = torch.zeros(ql, dtype=torch.int32, device=dev)
        kvl = torch.arange(ctx - ql + 1, ctx + 1, dtype=torch.int32, device=dev)
        ms_abs = _time(lambda: M.mla_attention(q_full, cache, bt, rows, kvl, scale, max_kvlen=ctx), max(2, iters // 4))
        return {"case": case, "ms": ms, "tflops_attn_plus_up": (attn_fl + up_fl) / ms / 1e9,
                "ms_absorbed_attention_only": ms_abs, "speedup_vs_absorbed": ms_abs / ms}
    if case in ("moe_decode", "moe_prefill"):
        # one expert-parallel shard of a DeepSeek-V3 layer: 32 local experts,
        # hidden 7168, expert width 2048; tokens x 8 slots spread over them
        from infera_b200.models.moe import MoELayer

        T = 64 if case == "moe_decode" else 2048
        E, H, F, k = 32, 7168, 2048, 8
        layer = MoELayer(H, F, E, k, device=dev, seed=0)
        x = torch.randn(T, H, device=dev, generator=g).to(bf)
        ids = torch.randint(0, E, (T, k), device=dev, dtype=torch.int32, generator=g)
        wts = torch.full((T, k), 1.0 / k, device=dev)
        ms = _time(lambda: layer.forward(x, ids, wts), iters)
        active = int(torch.unique(ids).numel())
        by = active * 3 * F * H * 2
        fl = 2 * T * k * 3 * F * H
        return {"case": case, "ms": ms, "gbs": by / ms / 1e6, "tflops": fl / ms / 1e9, "active_experts": active,
                "weight_bytes": by}
    if case in ("kv_push", "kv_push_local"):
        # 512 pages x 32 layers x (K, V) of an 8-KV-head x 128 cache: 1 GiB per push
        L, H, n = 32, hkv * D, 512
        src_dev = torch.device("cuda", 0)
        dst_dev = torch.device("cuda", 1 if case == "kv_push" else 0)
        slots = 2 * n * 16
        sk = torch.randn(L, slots, H, device=src_dev, generator=g).to(bf)
        sv = torch.randn(L, slots, H, device=src_dev, generator=g).to(bf)
        with torch.cuda.device(dst_dev):
            dk = torch.zeros(L, slots, H, dtype=bf, device=dst_dev)
            dv = torch.zeros(L, slots, H, dtype=bf, device=dst_dev)
        if dst_dev != src_dev:
            from infera_b200.ops import _native

            _native.check(_native.kernels().ib_enable_peer_access(dst_dev.index), "enable peer access")
        sp = torch.randperm(2 * n, device=src_dev)[:n].to(torch.int32)
        dp = torch.randperm(2 * n, device=src_dev)[:n].to(torch.int32)
        fn = lambda: K.kv_push_pages(sk, sv, dk.data_ptr(), dv.data_ptr(), sp, dp, dst_slots=slots)  # noqa: E731
        ms = _time(fn, iters)
        torch.cuda.synchronize(dst_dev)
        idx = (dp.long()[:, None] * 16 + torch.arange(16, device=src_dev)).reshape(-1).to(dst_dev)
        sidx = (sp.long()[:, None] * 16 + torch.arange(16, device=src_dev)).reshape(-1)
        ok = torch.equal(dk[:, idx].cpu(), sk[:, sidx].cpu())
        by = 2 * n * 16 * L * H * 2
        return {"case": case, "ms": ms, "gbs": by / ms / 1e6, "bytes": by, "exact": ok,
                "frac_of_nvlink_770": round(by / ms / 1e6 / 770, 3) if case == "kv_push" else None}
    raise SystemExit(f"unknown case {case}")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="+")
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    for case in a.cases:
        res = run_case(case, a.iters)
        res["status"] = K.scratch().read_status()
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

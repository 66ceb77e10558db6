"""Time to first token on a KV-tier hit against full recompute, one engine
with its HBM KV pool capped so long prefixes spill to the host tier.

    python -m infera_b200.bench.tier_ttft [--model qwen3-32b] [--prefix 65536] [--hbm-kv-gb 40]
        [--host-gb 64] [--sessions 3]

Sessions each own a unique random prefix of ``--prefix`` tokens (the
``tiering-32b`` trace's shape). The run visits sessions 0..n-1 in order
(every first visit is a full prompt computation: the cold TTFT), which
pushes session 0's pages out of the capped HBM pool into the host tier,
then revisits the last session (its prefix still in HBM: HBM-hit TTFT) and
session 0 (its prefix promoted from the host tier: tier-hit TTFT), each
revisit adding a 512-token increment as the trace's turns do. TTFT is the
host time from ``add_request`` to the step that returns the first token
(every step ends by reading its sampled tokens back, so the host clock
sees the device finish). The host tier's capacity is clamped to half of
the machine's available memory. Prints one JSON line.

The reference reports the same comparison for its kvd tiers
(``bench/kvcache/kv_cache_cliff/README.md``).
"""

from __future__ import annotations

import argparse
import json
import time

import torch

from infera_b200.ops import kernels as K


def _mem_available_gib() -> float:
    try:
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemAvailable:"):
                    return int(ln.split()[1]) / (1 << 20)
    except OSError:
        pass
    return 8.0


def _ttft(eng, rid: str, prompt: list[int]) -> tuple[float, int]:
    from infera_b200.engine.request import SamplingParams

    dev = eng.device
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    eng.add_request(rid, prompt, SamplingParams(max_tokens=2, ignore_eos=True))
    first = None
    cached = 0
    while eng.has_unfinished():
        for o in eng.step():
            if o.request_id == rid and o.new_token_ids and first is None:
                first = time.perf_counter() - t0
                cached = o.num_cached_tokens
    return first, cached


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-32b")
    ap.add_argument("--prefix", type=int, default=65536)
    ap.add_argument("--increment", type=int, default=512)
    ap.add_argument("--sessions", type=int, default=3)
    ap.add_argument("--hbm-kv-gb", type=float, default=40.0, help="HBM KV pool cap (GB)")
    ap.add_argument("--host-gb", type=float, default=64.0, help="host tier capacity (GiB), clamped to RAM / 2")
    ap.add_argument("--tier", choices=("pinned", "host"), default="pinned",
                    help="pinned: page-locked arena of page slots (DMA both ways); host: store of packed blobs")
    ap.add_argument("--max-batched-tokens", type=int, default=8192)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)

    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.models.config import get_config

    mc = get_config(a.model)
    page_bytes = 16 * mc.num_layers * mc.num_kv_heads * mc.head_dim * 2 * 2
    num_pages = int(a.hbm_kv_gb * 1e9 // page_bytes)
    host_gib = min(a.host_gb, 0.5 * _mem_available_gib())
    cfg = EngineConfig(model=a.model, num_pages=num_pages, max_num_seqs=4, max_batched_tokens=a.max_batched_tokens,
                       use_cuda_graphs=False, kv_tier=f"{a.tier}:{host_gib:.2f}", seed=a.seed)
    t_init = time.time()
    eng = LLMEngine(cfg, device=a.device)
    init_s = time.time() - t_init
    g = torch.Generator().manual_seed(a.seed)
    V = mc.vocab
    prefixes = [torch.randint(0, V, (a.prefix,), generator=g).tolist() for _ in range(a.sessions)]
    inc = lambda: torch.randint(0, V, (a.increment,), generator=g).tolist()  # noqa: E731
    cold = []
    for i, p in enumerate(prefixes):
        t, _ = _ttft(eng, f"cold{i}", p + inc())
        cold.append(t)
    eng.tier.flush()
    last = a.sessions - 1
    hbm_t, hbm_cached = _ttft(eng, "hbm", prefixes[last] + inc())
    loads0 = eng.tier.stats.get("loads", 0)
    tier_t, tier_cached = _ttft(eng, "tier", prefixes[0] + inc())
    st = dict(eng.tier.stats)
    out = {
        "metric": "TTFT on a KV-tier hit vs full recompute (one engine, HBM KV pool capped)",
        "model": a.model, "prefix_tokens": a.prefix, "increment": a.increment, "hbm_kv_gb": a.hbm_kv_gb,
        "num_pages": num_pages, "host_tier": a.tier, "host_tier_gib": round(host_gib, 1),
        "kv_bytes_per_token": page_bytes // 16,
        "ttft_cold_s": [round(x, 3) for x in cold],
        "ttft_hbm_hit_s": round(hbm_t, 3), "hbm_hit_cached_tokens": hbm_cached,
        "ttft_tier_hit_s": round(tier_t, 3), "tier_hit_cached_tokens": tier_cached,
        "speedup_tier_hit_vs_cold": round(sum(cold) / len(cold) / tier_t, 2) if tier_t else None,
        "tier_loads": st.get("loads", 0) - loads0, "tier_stats": st, "init_s": round(init_s, 1),
        "promote_gbs": round(st.get("promoted", 0) * page_bytes * 16 / 16 / st["load_s"] / 1e9, 1)
        if st.get("load_s") else None,
        "kernel_status": K.scratch(eng.device).read_status_detail() if eng.device.type == "cuda" else 0,
        "timing": "host clock, each step synchronises on its sampled tokens", "data": "synthetic random tokens",
    }
    eng.tier.close()
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

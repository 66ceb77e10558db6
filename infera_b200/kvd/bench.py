"""L3 (NVMe tier) bench through the engine's real tier path.

Drives :class:`~infera_b200.engine.tiering.TierManager` - the same batched
gather + copy-out on save and chunked pinned double-buffer + scatter on
promote the engine uses - against a :class:`~infera_b200.kvd.store.HostStore`
whose host budget is tiny, so every saved page spills to the O_DIRECT
tablespace under ``--dir``. Reports:

* save: pages evicted from the KV cache until they are in the tablespace
  (GB/s of KV payload, per-batch latency p50 / p95);
* cold reload: the host copies are dropped and the KV pages zeroed, then the
  pages are promoted from the tablespace back into the cache (GB/s, per-load
  latency p50 / p95);
* round trip: every reloaded page equals what was saved, byte for byte.

``python -m infera_b200.kvd.bench --dir /mnt/nvme/l3-bench --total-gb 4
[--model llama-3.1-8b] [--device cuda:0] [--chunk-pages 32]``. Role of the
reference's ``infera/kvd/bench/l3_bench.py`` and ``probe.py`` (which drive
its engine connector the same way).
"""

from __future__ import annotations

import argparse
import json
import shutil
import time


def run(directory: str, total_gb: float = 1.0, model: str = "llama-3.1-8b", device: str = "cuda:0",
        chunk_pages: int = 32, batch_pages: int = 64, layers: int | None = None) -> dict:
    import torch

    from infera_b200.engine.tiering import TierManager
    from infera_b200.kvd.store import HostStore
    from infera_b200.kvd.tablespace import Tablespace
    from infera_b200.models.config import get_config
    from infera_b200.bench.slo import percentile

    cfg = get_config(model)
    L = layers or cfg.num_layers
    H = cfg.num_kv_heads * cfg.head_dim
    ps = 16
    page_bytes = 2 * L * ps * H * 2
    n_pages = max(batch_pages, int(total_gb * (1 << 30)) // page_bytes)
    n_pages -= n_pages % batch_pages
    dev = torch.device(device)
    slots = (batch_pages + 1) * ps
    k = torch.randn(L, slots, H, device=dev).to(torch.bfloat16)
    v = torch.randn(L, slots, H, device=dev).to(torch.bfloat16)
    l3 = Tablespace(directory, fsync=False)
    store = HostStore(64 << 20, l3=l3)            # host budget << data: everything lands on NVMe
    tm = TierManager(k, v, store, ps, staging_pages=batch_pages, load_chunk=chunk_pages, async_load=False)
    pages = list(range(batch_pages))
    truth: dict[int, torch.Tensor] = {}
    save_lat = []
    t0 = time.monotonic()
    for b in range(n_pages // batch_pages):
        # fresh content for this batch; remember one page of it for the round-trip check
        k.normal_()
        v.normal_()
        hashes = [(b << 20) + i + 1 for i in range(batch_pages)]
        if b % 8 == 0:
            ref = torch.empty(1, tm.elems, dtype=torch.bfloat16, device=dev)
            from infera_b200.ops import kernels as K

            K.kv_page_copy(k, v, ref, torch.tensor([3], dtype=torch.int32, device=dev), ps, gather=True,
                           page_major=True)
            truth[hashes[3]] = ref.cpu()
        tb = time.monotonic()
        for p, h in zip(pages, hashes):
            tm.on_evict(p, h)
        tm.flush()
        save_lat.append(time.monotonic() - tb)
    l3.checkpoint()
    save_s = time.monotonic() - t0
    saved = tm.stats["saved"]
    # cold reload: drop every host copy (they are on NVMe), zero the cache
    with store.lock:
        for key in list(store.entries):
            store._drop(key, spill=True)          # the last ones still in host memory go to NVMe too
    k.zero_()
    v.zero_()
    load_lat = []
    ok = True
    t0 = time.monotonic()
    for b in range(n_pages // batch_pages):
        hashes = [(b << 20) + i + 1 for i in range(batch_pages)]
        tb = time.monotonic()
        got = tm.load(pages, hashes)
        if dev.type == "cuda":
            torch.cuda.synchronize()
        load_lat.append(time.monotonic() - tb)
        if got != batch_pages:
            ok = False
        if hashes[3] in truth:
            chk = torch.empty(1, tm.elems, dtype=torch.bfloat16, device=dev)
            from infera_b200.ops import kernels as K

            K.kv_page_copy(k, v, chk, torch.tensor([3], dtype=torch.int32, device=dev), ps, gather=True,
                           page_major=True)
            ok = ok and torch.equal(chk.cpu(), truth[hashes[3]])
    load_s = time.monotonic() - t0
    tm.close()
    l3.close()
    gb = n_pages * page_bytes / 1e9
    return {"dir": directory, "model": model, "layers": L, "page_bytes": page_bytes, "pages": n_pages,
            "payload_gb": round(gb, 3), "saved": saved, "l3_io": "direct" if l3.direct else "buffered",
            "save_gbs": round(gb / save_s, 3), "save_batch_ms_p50": round(1000 * percentile(save_lat, 50), 2),
            "save_batch_ms_p95": round(1000 * percentile(save_lat, 95), 2),
            "reload_gbs": round(gb / load_s, 3), "reload_batch_ms_p50": round(1000 * percentile(load_lat, 50), 2),
            "reload_batch_ms_p95": round(1000 * percentile(load_lat, 95), 2), "round_trip_ok": ok}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="python -m infera_b200.kvd.bench")
    ap.add_argument("--dir", required=True)
    ap.add_argument("--total-gb", type=float, default=1.0)
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--chunk-pages", type=int, default=32)
    ap.add_argument("--batch-pages", type=int, default=64)
    ap.add_argument("--keep", action="store_true", help="keep the tablespace files afterwards")
    a = ap.parse_args(argv)
    try:
        res = run(a.dir, a.total_gb, a.model, a.device, a.chunk_pages, a.batch_pages, a.layers)
    finally:
        if not a.keep:
            shutil.rmtree(a.dir, ignore_errors=True)
    print(json.dumps(res))


if __name__ == "__main__":
    main()

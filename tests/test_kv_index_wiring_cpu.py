"""The tier-aware KV index end to end on CPU: an engine's device blocks and
tier moves translated by the engine-side feed into index events, the
router's plane subscribing to a worker that registers a kv block (and
dropping it when it leaves), the reconciler pulling the worker's snapshot
over HTTP, and the router's /v1/kv-stats, /v1/kv-index/match and
cache-view routes."""

import asyncio

import httpx
import torch
from fastapi import FastAPI

from infera_b200.bench.fleet import free_port
from infera_b200.common.discovery import InProcessRegistry
from infera_b200.common.worker_pool import KvRegistrationMetadata, WorkerInfo
from infera_b200.engine.kv_index_feed import KvIndexFeed
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.kv.hashing import hash_token_blocks
from infera_b200.kv.plane import KvIndexPlane
from infera_b200.kv.publisher import KvIndexPublisher
from infera_b200.kv.types import Tier
from infera_b200.utils.hashing import chain_hashes


def _prompt(seed, n):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1024, (n,), generator=g).tolist()


def test_feed_translates_device_blocks_and_tier_moves():
    batches = []
    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=64), device="cpu")
    feed = KvIndexFeed("w0", "m", "c", 16, sink=batches.append)
    eng.attach_kv_index(feed)
    p = _prompt(1, 70)                       # 4 full pages + 6 tokens (+ 2 generated)
    eng.generate([p], SamplingParams(max_tokens=2, ignore_eos=True))
    feed.flush()
    want = hash_token_blocks(p, 16)          # the index's own keys of the prompt's full pages
    idx = feed._local
    m = idx.find_matches("m", "c", want)
    assert m["w0"].device() == 4
    assert batches and batches[0].events[0].kind == "stored"
    # a page saved to the host tier, then evicted from the device: still held (host)
    h = chain_hashes(p, 16)
    feed.on_tier_event("stored", Tier.HOST, h[:4])
    feed.on_engine_event("BlockRemoved", {"block_hashes": h[:4], "medium": "GPU"})
    m = idx.find_matches("m", "c", want)
    assert m["w0"].device() == 0 and m["w0"].by_tier[Tier.HOST] == 4
    assert feed.tiers_of(h[0]) == {Tier.HOST}
    feed.on_tier_event("removed", Tier.HOST, h[2:4])
    assert idx.find_matches("m", "c", want)["w0"].by_tier[Tier.HOST] == 2
    snap = feed.snapshot()
    assert snap["publisher"] == "w0" and snap["chains"][0]["tier"] == "host"


def test_router_plane_follows_registry_and_reconciles():
    async def go():
        ep = f"tcp://127.0.0.1:{free_port()}"
        pub = KvIndexPublisher(ep)
        feed = KvIndexFeed("w0:1", "m", "c", 16, sink=pub)
        snap_calls = []

        async def fetch(target):
            snap_calls.append(target)
            return feed.snapshot()

        plane = KvIndexPlane(fetch=fetch, period_s=3600)
        await plane.start()
        reg = InProcessRegistry()
        reg.on_worker_added(plane.on_worker_added)
        reg.on_worker_removed(plane.on_worker_removed)
        kv = KvRegistrationMetadata(engine_block_size=16, index_block_size=16, tokenizer="byte",
                                    tokenizer_digest="c", tokenizer_canary=[1], events_endpoint=ep,
                                    snapshot_endpoint="http://w0:1", tiers=["device", "host"])
        reg.register(WorkerInfo("w0:1", "http://w0:1", "m", kv=kv).to_payload())
        p = _prompt(2, 64)
        want = hash_token_blocks(p, 16)
        hashes = chain_hashes(p, 16)
        for _ in range(60):                   # slow joiner: publish until the subscriber sees it
            feed.on_engine_event("AllBlocksCleared", {})
            feed.on_engine_event("BlockStored", {"block_hashes": hashes, "parent_block_hash": None,
                                                 "token_ids": p, "block_size": 16})
            feed.flush()
            await asyncio.sleep(0.05)
            if plane.index.find_matches("m", "c", want):
                break
        got = plane.index.find_matches("m", "c", want)["w0:1"].device()
        # routes
        from infera_b200.kv.api import index_router, stats_router

        app = FastAPI()
        app.include_router(stats_router(plane))
        app.include_router(index_router(plane.index))
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app), base_url="http://t") as c:
            st = (await c.get("/v1/kv-stats")).json()
            mt = (await c.post("/v1/kv-index/match", json={"model": "m", "compat": "c", "token_ids": p,
                                                           "block_size": 16})).json()
        # a lost event is repaired by the reconciler's snapshot
        feed._pending.clear()
        feed.on_tier_event("stored", Tier.HOST, hashes)
        feed._pending.clear()
        assert await plane.reconciler.reconcile_once() == 1
        tiers = plane.index.tier_counts("w0:1")
        reg.deregister("w0:1")
        await asyncio.sleep(0.05)
        left = plane.index.tier_counts("w0:1")
        await plane.stop()
        pub.close()
        return got, st, mt, snap_calls, tiers, left

    got, st, mt, calls, tiers, left = asyncio.run(go())
    assert got == 4
    assert st["index"]["trees"] == 1 and st["subscribers"]["endpoints"]
    assert mt["matches"]["w0:1"]["device"] == 4
    assert calls and calls[0][0] == "http://w0:1" and calls[0][1] == "m" and calls[0][2] == "c"
    assert tiers == {"device": 4, "host": 4}
    assert left == {}

"""The tier-aware KV index package: hashing, radix tree with tiers and
optimistic nodes, engine-block probe, wire formats, ZMQ publish -> single
writer, snapshot reconciliation and the match API."""

import asyncio

import httpx
from fastapi import FastAPI

from infera_b200.bench.fleet import free_port
from infera_b200.kv.api import index_router
from infera_b200.kv.compat_key import compat_key
from infera_b200.kv.families import family_of
from infera_b200.kv.hashing import hash_prompt, hash_token_blocks, lora_hash
from infera_b200.kv.index import KVIndex
from infera_b200.kv.probe import KvEventProbe
from infera_b200.kv.publisher import KvIndexPublisher
from infera_b200.kv.types import MmRun, Tier
from infera_b200.kv.wire import decode_batch, encode_batch, snapshot_chains, snapshot_json
from infera_b200.kv.writer import KvIndexSubscriber, KvIndexWriter, SnapshotReconciler

TOK = list(range(1000, 1256))


def test_hashing_and_keys():
    a = hash_token_blocks(TOK, 64)
    assert len(a) == 4 and a == hash_token_blocks(TOK + [1, 2], 64)
    assert hash_token_blocks(TOK, 64, lora=lora_hash("x")) != a
    assert [k.block_hash for k in hash_token_blocks(TOK[64:128], 64)] == [a[1].block_hash]  # content hash
    assert hash_token_blocks(TOK[64:128], 64)[0].sequence_hash != a[1].sequence_hash     # chained
    mm = hash_prompt(TOK, 64, mm_runs=[MmRun(70, 10, 42)])
    assert mm[0] == a[0] and mm[1] != a[1]
    assert family_of("meta-llama/Llama-3.1-8B-Instruct") == "llama-3" and family_of("Qwen3-32B") == "qwen3"
    assert compat_key("llama-3.1-8b", "d", 64) != compat_key("llama-3.1-8b", "d", 64, role="decode")


def test_index_tiers_removal_and_optimistic():
    ix = KVIndex()
    q = hash_token_blocks(TOK, 64)
    k0, k1 = ("m", "c", "p0"), ("m", "c", "p1")
    ix.apply_stored(k0, q[:2], None, Tier.DEVICE)
    ix.apply_stored(k0, q[2:], q[1].sequence_hash, Tier.HOST)
    ix.apply_stored(k1, q[:1], None, Tier.DEVICE)
    m = ix.find_matches("m", "c", q)
    assert m["p0"].by_tier[Tier.DEVICE] == 2 and m["p0"].by_tier[Tier.HOST] == 4 and m["p0"].best() == 4
    assert m["p1"].device() == 1
    # evicted from the device tier: block 1 stays in host (spilled)
    ix.apply_stored(k0, [q[1]], q[0].sequence_hash, Tier.HOST)
    ix.apply_removed(k0, [q[1].sequence_hash], Tier.DEVICE)
    assert ix.find_matches("m", "c", q)["p0"].by_tier.get(Tier.DEVICE) == 1
    # gone from every tier: the subtree goes too
    ix.apply_removed(k0, [q[1].sequence_hash], None)
    assert ix.find_matches("m", "c", q)["p0"].best() == 1
    # unknown parent: dropped
    assert ix.apply_stored(k1, q[3:], 12345, Tier.DEVICE) == 0 and ix.stats.dropped_unknown_parent == 1
    # optimistic placement expires unless confirmed
    ix.insert_optimistic(k1, q, ttl_ms=50)
    assert ix.find_matches("m", "c", q)["p1"].device() == 4
    assert ix.evict_expired(now=10**15) >= 3
    assert ix.find_matches("m", "c", q)["p1"].device() == 1


def test_probe_coalesces_engine_blocks_and_snapshot_roundtrip():
    batches = []
    pr = KvEventProbe("p0", "m", "c", engine_block=16, index_block=64, sink=batches.append)
    ehs = list(range(100, 116))  # 16 engine blocks = 4 index blocks
    pr.on_sequence_cached(TOK, ehs[:6])   # 1 full index block resident
    pr.on_sequence_cached(TOK, ehs)       # the rest
    pr.flush()
    ix = KVIndex()
    w = KvIndexWriter(ix)
    for b in batches:
        w.apply(decode_batch(encode_batch(b)))
    q = hash_token_blocks(TOK, 64)
    assert ix.find_matches("m", "c", q)["p0"].device() == 4
    pr.on_engine_blocks_evicted([109])    # inside index block 2
    w.apply(decode_batch(encode_batch(pr.flush())))
    assert ix.find_matches("m", "c", q)["p0"].device() == 2
    snap = snapshot_json("p0", "m", "c", pr.chains())
    ix2 = KVIndex()
    ix2.replace(("m", "c", "p0"), snapshot_chains(snap))
    assert ix2.find_matches("m", "c", q)["p0"].device() == 2


def test_zmq_publish_writer_reconcile_and_api():
    async def go():
        ix = KVIndex()
        w = KvIndexWriter(ix)
        w.start()
        sub = KvIndexSubscriber(w)
        ep = f"tcp://127.0.0.1:{free_port()}"
        pub = KvIndexPublisher(ep)
        sub.add(ep)
        pr = KvEventProbe("p0", "m", "c", 16, 64, sink=pub)
        q = hash_token_blocks(TOK, 64)
        for _ in range(50):  # slow joiner: publish until the subscriber sees it
            pr.on_cleared()
            pr.on_sequence_cached(TOK, list(range(16)))
            pr.flush()
            await asyncio.sleep(0.05)
            if ix.find_matches("m", "c", q):
                break
        assert ix.find_matches("m", "c", q)["p0"].device() == 4
        # a removal that never arrives is repaired by the reconciler
        pr._pending.clear()
        pr.on_engine_blocks_evicted([0])
        pr._pending.clear()
        rec = SnapshotReconciler(ix, lambda: ["p0"],
                                 lambda url: asyncio.sleep(0, snapshot_json("p0", "m", "c", pr.chains())))
        assert await rec.reconcile_once() == 1
        assert "p0" not in ix.find_matches("m", "c", q)
        app = FastAPI()
        app.include_router(index_router(ix))
        pr.on_sequence_cached(TOK, list(range(16)))
        w.apply(pr.flush())
        async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app), base_url="http://t") as c:
            r = await c.post("/v1/kv-index/match", json={"model": "m", "compat": "c", "token_ids": TOK,
                                                         "block_size": 64})
            st = await c.get("/v1/kv-index/stats")
        await sub.stop()
        await w.stop()
        pub.close()
        return r.json(), st.json()

    res, st = asyncio.run(go())
    assert res["query_blocks"] == 4 and res["matches"]["p0"]["device"] == 4
    assert st["trees"] == 1

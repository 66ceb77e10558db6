"""KV tier daemon: wire framing, seqlock arena, priority LRU with L3 spill and
promotion, journaled tablespace restart, and the UDS server with arena fd
passing and zero-copy save leases."""

import asyncio
import os

import pytest

from infera_b200.kvd import wire as W
from infera_b200.kvd.client import KvdClient
from infera_b200.kvd.server import KvdServer
from infera_b200.kvd.shared_arena import ArenaView, SharedArena
from infera_b200.kvd.store import HostStore
from infera_b200.kvd.tablespace import Tablespace


def test_wire_roundtrip():
    for msg in [W.Hello("c", 1, True), W.Set(b"k" * 8, b"v" * 100, "long", ttl_seconds=5.0),
                W.BatchGetSharedResponse([(16, 4, 2), None]), W.HelloAck("s", 1, (1024, 64, 7)),
                W.StatsResponse(1, 2, 3, 4, 5, 6, 7, 8, 9)]:
        raw = W.encode(msg)
        assert int.from_bytes(raw[:4], "big") == len(raw) - 4
        assert W.decode_body(raw[4:]) == msg


def test_arena_seqlock():
    a = SharedArena(4, 4096)
    s = a.alloc()
    v = a.write(s, b"hello")
    view = ArenaView(os.dup(a.fd), a.size, a.slot_size)
    assert view.read(a.payload_offset(s), v) == b"hello"
    v2 = a.write(s, b"world!")
    assert view.read(a.payload_offset(s), v) is None          # rewritten: reader sees a miss
    assert view.read(a.payload_offset(s), v2) == b"world!"
    a.begin_write(s)                                          # writer in progress: odd version
    assert view.read(a.payload_offset(s), None, retries=3) is None
    view.close()
    a.close()


def test_priority_lru_spill_and_promote(tmp_path):
    l3 = Tablespace(str(tmp_path / "l3"), container_bytes=1 << 20, slot_bytes=1 << 12, fsync=False)
    st = HostStore(0, arena=SharedArena(3, 8192), l3=l3)
    assert st.set(b"a" * 8, b"A" * 100, "long")
    assert st.set(b"b" * 8, b"B" * 100, "short")
    assert st.set(b"c" * 8, b"C" * 100, "short")
    assert st.set(b"d" * 8, b"D" * 100, "short")       # evicts the LRU short entry (b) to L3
    assert st.tier(b"b" * 8) == "file" and st.tier(b"a" * 8) == "ram"
    assert not st.set(b"e" * 8, b"E" * 100, "none") or st.tier(b"a" * 8) == "ram"
    assert st.get(b"b" * 8) == b"B" * 100               # promoted back from L3
    assert st.stats["promotions"] == 1
    st2 = HostStore(0, arena=SharedArena(1, 8192))
    assert st2.set(b"x" * 8, b"X", "long")
    assert not st2.set(b"y" * 8, b"Y", "short")         # never displaces a higher priority entry
    assert st2.stats["rejected"] == 1


def test_tablespace_restart_and_torn_journal(tmp_path):
    root = str(tmp_path / "ts")
    ts = Tablespace(root, container_bytes=1 << 20, slot_bytes=1 << 12)
    assert ts.put(b"k1" * 4, b"1" * 5000, "long")
    assert ts.put(b"k2" * 4, b"2" * 100)
    ts.checkpoint()
    assert ts.put(b"k3" * 4, b"3" * 9000)
    assert ts.delete(b"k2" * 4)
    ts.close()
    with open(os.path.join(root, "index.log"), "ab") as f:
        f.write(b"\x10\x00\x00\x00garbage")           # torn tail of a crashed append
    ts = Tablespace(root, container_bytes=1 << 20, slot_bytes=1 << 12)
    assert ts.get(b"k1" * 4) == b"1" * 5000 and ts.get(b"k3" * 4) == b"3" * 9000
    assert ts.get(b"k2" * 4) is None and len(ts) == 2
    ts.close()


def test_daemon_roundtrip_with_arena_and_lease(tmp_path):
    path = str(tmp_path / "kvd.sock")
    l3 = Tablespace(str(tmp_path / "l3"), container_bytes=1 << 20, slot_bytes=1 << 12, fsync=False)
    store = HostStore(0, arena=SharedArena(8, 1 << 14), l3=l3)

    async def go():
        srv = KvdServer(path, store)
        await srv.start()
        plain = KvdClient(path)
        await plain.connect()
        assert await plain.set(b"k" * 8, b"value", "long")
        assert await plain.get(b"k" * 8) == b"value"
        shared = KvdClient(path)
        await shared.connect(shared_arena=True)
        assert shared.arena is not None
        assert await shared.get(b"k" * 8) == b"value"        # read in place from the arena
        lease = await shared.set_lease(b"z" * 8, 64, "short")
        assert lease.ok
        assert await shared.commit_set(lease, b"Z" * 64)
        assert await plain.get(b"z" * 8) == b"Z" * 64
        assert await plain.exists([b"k" * 8, b"q" * 8]) == [True, False]
        t = await plain.lookup_tier(b"k" * 8)
        assert t.tier == "ram"
        st = await plain.stats()
        assert st.entries == 2 and st.hits_total >= 3
        # a client that disconnects with an open lease gives the slot back
        free0 = store.arena.free_slots()
        c3 = KvdClient(path)
        await c3.connect(shared_arena=True)
        lease = await c3.set_lease(b"w" * 8, 32)
        assert store.arena.free_slots() == free0 - 1
        await c3.close()
        for _ in range(50):
            if store.arena.free_slots() == free0:
                break
            await asyncio.sleep(0.02)
        assert store.arena.free_slots() == free0
        assert await plain.clear() == 2
        await plain.close()
        await shared.close()
        await srv.stop()

    asyncio.run(go())

"""More KV tier daemon behaviour: TTL expiry, overwrite, zero-copy
reservation commit / cancel, capacity accounting, clear; tablespace
multi-slot values, overwrite, delete + restart, checkpoint + journal
replay, space reuse after delete, LRU eviction by retention."""

import time

import pytest

from infera_b200.kvd.shared_arena import SharedArena
from infera_b200.kvd.store import HostStore
from infera_b200.kvd.tablespace import Tablespace


def test_ttl_expiry_and_overwrite():
    st = HostStore(1 << 20)
    assert st.set(b"k" * 8, b"v1", "short", ttl=0.05)
    assert st.get(b"k" * 8) == b"v1"
    time.sleep(0.08)
    assert st.get(b"k" * 8) is None and not st.exists(b"k" * 8)
    assert st.set(b"k" * 8, b"v2", "long")
    assert st.set(b"k" * 8, b"v3", "long")              # overwrite keeps one entry
    assert st.get(b"k" * 8) == b"v3"
    assert st.clear() >= 1 and st.get(b"k" * 8) is None


def test_reservation_commit_and_cancel():
    arena = SharedArena(2, 4096)
    st = HostStore(0, arena=arena)
    r = st.reserve(b"a" * 8, 100, "long")
    assert r is not None
    slot, reserved = r[0], r[1]
    arena.write(slot, b"Z" * 100)
    st.commit(b"a" * 8, slot, 100, reserved, "long", None)
    assert st.get(b"a" * 8) == b"Z" * 100
    r2 = st.reserve(b"b" * 8, 100, "long")
    assert r2 is not None
    st.cancel(r2[0], r2[1])                              # cancelled: the slot is reusable
    assert st.get(b"b" * 8) is None
    assert st.set(b"c" * 8, b"C" * 10, "long")


def test_capacity_rejects_oversized_values():
    st = HostStore(1000)
    assert not st.set(b"x" * 8, b"X" * 5000, "long")
    assert st.set(b"y" * 8, b"Y" * 600, "short")
    assert st.set(b"z" * 8, b"Z" * 600, "short")         # evicts y (no L3: dropped)
    assert st.get(b"y" * 8) is None and st.get(b"z" * 8) == b"Z" * 600


def _ts(root, **kw):
    kw.setdefault("container_bytes", 1 << 20)
    kw.setdefault("slot_bytes", 1 << 12)
    return Tablespace(str(root), fsync=False, **kw)


def test_tablespace_multislot_overwrite_delete_restart(tmp_path):
    ts = _ts(tmp_path / "ts")
    big = bytes(range(256)) * 70                         # 17920 B: five 4 KiB slots
    assert ts.put(b"big00000", big)
    assert ts.put(b"small000", b"s" * 10)
    assert ts.get(b"big00000") == big
    assert ts.put(b"small000", b"t" * 20)                # overwrite
    assert ts.delete(b"big00000") and not ts.delete(b"big00000")
    used = ts.bytes_used()
    ts.close()
    ts2 = _ts(tmp_path / "ts")                           # journal replay
    assert ts2.get(b"big00000") is None and ts2.get(b"small000") == b"t" * 20
    assert ts2.bytes_used() == used
    # freed space is reused
    for i in range(50):
        assert ts2.put(f"k{i:07d}".encode(), big)
    ts2.checkpoint()
    ts2.close()
    ts3 = _ts(tmp_path / "ts")                           # snapshot + (empty) journal
    assert all(ts3.get(f"k{i:07d}".encode()) == big for i in range(0, 50, 7))
    ts3.close()


def test_tablespace_evicts_lowest_priority_first(tmp_path):
    ts = _ts(tmp_path / "ts2")
    for i in range(4):
        ts.put(f"s{i:07d}".encode(), b"x" * 4096, "short")
        ts.put(f"l{i:07d}".encode(), b"x" * 4096, "long")
    prio = {"none": 0, "short": 1, "long": 2}
    freed = ts.evict_lru(3 * 4096, lambda r: prio.get(r, 1))
    assert freed >= 3 * 4096
    longs = sum(ts.get(f"l{i:07d}".encode()) is not None for i in range(4))
    assert longs == 4
    ts.close()


def test_tablespace_rejects_bad_geometry(tmp_path):
    with pytest.raises(ValueError):
        Tablespace(str(tmp_path / "bad"), container_bytes=10000, slot_bytes=4096)


def test_l3_bench_round_trip_through_the_tier_path(tmp_path):
    """The L3 bench drives the engine's tier manager: pages saved through the
    host store land on the tablespace and come back byte for byte."""
    from infera_b200.kvd.bench import run

    res = run(str(tmp_path / "l3"), total_gb=0.01, device="cpu", layers=2, batch_pages=8, chunk_pages=4)
    assert res["round_trip_ok"] and res["saved"] == res["pages"] and res["reload_gbs"] > 0

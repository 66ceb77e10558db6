"""kvd L3 extras: size-classed and striped tablespaces, storage
classification from a fake mount table, the self-check, the per-file L3
reaper and the layer-wise loader (CPU path)."""

import collections
import os

import torch

from infera_b200.engine.l3_reaper import L3FileReaper, retention_of
from infera_b200.engine.layerwise_load import LayerwiseLoader
from infera_b200.kvd.multipool import MultiPoolTablespace, StripedTablespace
from infera_b200.kvd.storage import classify, selfcheck


def test_multipool_routes_by_size(tmp_path):
    mp = MultiPoolTablespace(str(tmp_path), slot_sizes=(4096, 65536), container_bytes=1 << 20, max_slots=4,
                             fsync=False, direct_io=False)
    small, big = os.urandom(3000), os.urandom(100_000)
    assert mp.put(b"s", small) and mp.put(b"b", big)
    assert mp.pool_for(len(small)) == 0 and mp.pool_for(len(big)) == 1
    assert mp.get(b"s") == small and mp.get(b"b") == big
    assert mp.put(b"s", big) and mp.get(b"s") == big and len(mp) == 2  # moved pools
    assert mp.delete(b"b") and b"b" not in mp
    mp.close()


def test_striped_parallel_io(tmp_path):
    roots = [str(tmp_path / f"d{i}") for i in range(3)]
    st = StripedTablespace(roots, container_bytes=1 << 20, slot_bytes=4096, fsync=False, direct_io=False)
    items = [(f"k{i}".encode(), os.urandom(5000)) for i in range(30)]
    assert all(st.put_many(items))
    assert st.get_many([k for k, _ in items]) == [v for _, v in items]
    assert len({st.shard_of(k) for k, _ in items}) == 3 and len(st) == 30
    st.close()


def test_classify(tmp_path):
    mounts = tmp_path / "mounts"
    mounts.write_text("/dev/nvme0n1p1 /data xfs rw 0 0\n"
                      "srv:/x /nfs nfs4 rw,wsize=65536 0 0\n"
                      "overlay / overlay rw 0 0\n"
                      "tmpfs /dev/shm tmpfs rw 0 0\n")
    c = classify("/data/kv", str(mounts), str(tmp_path))
    assert c.kind == "nvme" and c.io_mode == "direct"
    n = classify("/nfs/a", str(mounts), str(tmp_path))
    assert n.kind == "network" and n.io_mode == "buffered" and any("wsize" in w for w in n.warnings)
    assert classify("/other", str(mounts), str(tmp_path)).kind == "overlay"
    assert classify("/dev/shm/x", str(mounts), str(tmp_path)).io_mode == "buffered"
    res = selfcheck(str(tmp_path / "sc"), mib=2)
    assert res["write_gbs"] > 0 and res["read_gbs"] > 0


def test_reaper_budget_priority_and_floor(tmp_path):
    d = tmp_path / "l3"
    d.mkdir()
    for i, ret in enumerate(["long", "none", "short", "long", "ephemeral"]):
        p = d / f"c{i}.{ret}.kvcache"
        p.write_bytes(b"x" * 1000)
        os.utime(p, (1000 + i, 1000 + i))
    Usage = collections.namedtuple("Usage", "total used free")
    free = [10_000_000]
    r = L3FileReaper(str(d), budget_bytes=3000, disk_usage=lambda p: Usage(0, 0, free[0]))
    freed = r.reap()
    left = sorted(os.listdir(d))
    assert freed == 2000 and left == ["c0.long.kvcache", "c2.short.kvcache", "c3.long.kvcache"]
    assert retention_of("a.long.kvcache") == "long" and retention_of("a.kvcache") == "short"
    # free-space floor: a full disk reaps even under budget
    free[0] = 500
    r.floor = 2000
    r.budget = None
    r.reap(0)
    assert len(os.listdir(d)) == 1
    # clamp: budget cannot exceed what the disk holds above the floor
    r.budget = 10**12
    assert r.startup_budget_clamp() <= 1000 + 500
    r.write_with_reap("new.long.kvcache", b"y" * 10)
    assert (d / "new.long.kvcache").exists()


def test_layerwise_loader_cpu():
    ld = LayerwiseLoader(num_layers=3, buf_bytes=3 * 16, pool_size=1, device="cpu")
    buf = ld.staging()
    buf.copy_(torch.arange(48, dtype=torch.uint8))
    dsts = [torch.zeros(16, dtype=torch.uint8) for _ in range(3)]
    ld.load(buf, dsts, 16)
    ld.wait_layer(1)
    ld.synchronize()
    assert torch.equal(dsts[2], torch.arange(32, 48, dtype=torch.uint8))
    assert len(ld.free) == 1

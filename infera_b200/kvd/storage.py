"""What kind of storage an L3 path sits on, and whether it is fast enough.

``classify(path)`` reads the mount table for the path's filesystem and the
block device's ``queue/rotational`` flag: local NVMe / SSD -> O_DIRECT I/O,
NFS / tmpfs / overlay -> buffered I/O (O_DIRECT there is either refused or
slower), spinning disks -> buffered with a warning. NFS mounts with a
``wsize`` under 1 MiB get a warning (large chunks then fragment).
``selfcheck(path)`` writes and reads a few MiB and reports throughput, with
a warning below a floor. Roles of ``infera/kvd/storage_classify.py`` and
``infera/kvd/storage_selfcheck.py``.
"""

from __future__ import annotations

import mmap
import os
import time
from dataclasses import dataclass, field


@dataclass
class StorageClass:
    path: str
    fstype: str
    device: str | None
    kind: str            # nvme / ssd / hdd / network / memory / overlay / unknown
    io_mode: str         # direct / buffered
    warnings: list[str] = field(default_factory=list)


def _mounts(mounts_file: str = "/proc/mounts") -> list[tuple[str, str, str, str]]:
    out = []
    try:
        with open(mounts_file) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 4:
                    out.append((parts[0], parts[1], parts[2], parts[3]))
    except OSError:
        pass
    return out


def _mount_of(path: str, mounts) -> tuple[str, str, str, str] | None:
    path = os.path.realpath(path)
    best = None
    for dev, mnt, fstype, opts in mounts:
        if path == mnt or path.startswith(mnt.rstrip("/") + "/") or mnt == "/":
            if best is None or len(mnt) > len(best[1]):
                best = (dev, mnt, fstype, opts)
    return best


def _rotational(dev: str, sys_block: str = "/sys/block") -> bool | None:
    name = os.path.basename(dev)
    cands = [name]
    base = name.rstrip("0123456789")
    if name.startswith("nvme") and "p" in name:
        cands.append(name.rsplit("p", 1)[0])
    elif base != name:
        cands.append(base)
    for c in cands:
        try:
            with open(os.path.join(sys_block, c, "queue", "rotational")) as f:
                return f.read().strip() == "1"
        except OSError:
            continue
    return None


def classify(path: str, mounts_file: str = "/proc/mounts", sys_block: str = "/sys/block") -> StorageClass:
    m = _mount_of(path, _mounts(mounts_file))
    if m is None:
        return StorageClass(path, "unknown", None, "unknown", "buffered", ["mount not found"])
    dev, _mnt, fstype, opts = m
    warns = []
    if fstype.startswith("nfs") or fstype in ("cifs", "smb3", "lustre", "ceph", "fuse.sshfs"):
        kind, mode = "network", "buffered"
        for o in opts.split(","):
            if o.startswith("wsize="):
                try:
                    if int(o.split("=")[1]) < (1 << 20):
                        warns.append(f"NFS wsize {o.split('=')[1]} < 1 MiB: large chunks will fragment")
                except ValueError:
                    pass
    elif fstype in ("tmpfs", "ramfs"):
        kind, mode = "memory", "buffered"
        warns.append("L3 on memory-backed storage duplicates the host tier")
    elif fstype in ("overlay", "overlayfs", "aufs"):
        kind, mode = "overlay", "buffered"
        warns.append("L3 on a container overlay filesystem: mount a real volume")
    else:
        rot = _rotational(dev, sys_block)
        if "nvme" in dev:
            kind, mode = "nvme", "direct"
        elif rot is False:
            kind, mode = "ssd", "direct"
        elif rot is True:
            kind, mode = "hdd", "buffered"
            warns.append("L3 on a rotational disk")
        else:
            kind, mode = "unknown", "buffered"
    return StorageClass(path, fstype, dev, kind, mode, warns)


def selfcheck(path: str, mib: int = 16, floor_gbs: float = 0.5) -> dict:
    os.makedirs(path, exist_ok=True)
    f = os.path.join(path, ".l3_selfcheck")
    buf = mmap.mmap(-1, mib << 20)
    buf.write(os.urandom(1 << 16) * ((mib << 20) >> 16))
    t0 = time.perf_counter()
    fd = os.open(f, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o644)
    try:
        os.write(fd, buf)
        os.fsync(fd)
    finally:
        os.close(fd)
    tw = time.perf_counter() - t0
    t0 = time.perf_counter()
    fd = os.open(f, os.O_RDONLY)
    try:
        while os.read(fd, 1 << 20):
            pass
    finally:
        os.close(fd)
    tr = time.perf_counter() - t0
    os.unlink(f)
    w, r = (mib / 1024) / max(tw, 1e-9), (mib / 1024) / max(tr, 1e-9)
    res = {"write_gbs": round(w, 3), "read_gbs": round(r, 3), "warnings": []}
    if w < floor_gbs:
        res["warnings"].append(f"L3 write throughput {w:.2f} GB/s below {floor_gbs} GB/s")
    return res

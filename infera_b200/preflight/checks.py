"""Node probes of the preflight (one B200 box).

Every probe returns ``(data, findings)``: ``data`` is what it measured or
read, ``findings`` are :class:`Finding` s at level info / warn / fail. GPU
state is read through NVML with query calls only (nothing here changes a
clock, a power limit or any other GPU setting). Probes that need what the
node lacks (no GPU, no NVML, no torch) skip with an info finding, so a
host-only run still works.

Roles of the reference's ``infera/tools/preflight/{host,gpu,storage}/*.py``;
the RDMA / Mooncake / MoRI probes have no counterpart here (PD transfers run
over NVLink inside one box, checked by the P2P matrix).
"""

from __future__ import annotations

import os
import platform
import resource
import statistics
import time
from dataclasses import asdict, dataclass, field


@dataclass
class Finding:
    check: str
    level: str          # info / warn / fail
    message: str
    data: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        return asdict(self)


LEVELS = {"info": 0, "warn": 1, "fail": 2}

# B200 floors, well under what this pool's B200s measure (bf16 GEMM ~1675
# TFLOP/s burst, copy ~6400 GB/s, NVLink peer copy ~770 GB/s per direction):
# a GPU below them is broken or throttled, not just slower.
B200_GEMM_MIN_TFLOPS = 1100.0
B200_HBM_MIN_GBS = 5000.0
B200_P2P_MIN_GBS = 500.0
B200_NVLINKS = 18
SLOW_FRAC = 0.9      # relative outlier: below this fraction of the node median


# ---------------------------------------------------------------- host
def host_info(proc: str = "/proc", sys_node: str = "/sys/devices/system/node") -> tuple[dict, list[Finding]]:
    f: list[Finding] = []
    d = {"hostname": platform.node(), "kernel": platform.release(), "cpus": os.cpu_count()}
    try:
        with open(os.path.join(proc, "cpuinfo")) as fh:
            for line in fh:
                if line.startswith("model name"):
                    d["cpu_model"] = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        with open(os.path.join(proc, "meminfo")) as fh:
            for line in fh:
                k, _, v = line.partition(":")
                if k in ("MemTotal", "MemAvailable", "HugePages_Total"):
                    d[k] = int(v.split()[0])
    except OSError:
        pass
    try:
        d["numa_nodes"] = sorted(int(x[4:]) for x in os.listdir(sys_node) if x.startswith("node") and x[4:].isdigit())
    except OSError:
        d["numa_nodes"] = []
    soft, hard = resource.getrlimit(resource.RLIMIT_MEMLOCK)
    d["memlock_soft"] = soft
    d["memlock_hard"] = hard
    if soft != resource.RLIM_INFINITY and soft < (64 << 30):
        f.append(Finding("host.memlock", "warn",
                         f"RLIMIT_MEMLOCK is {soft >> 20} MiB: pinned host KV tiers and staging buffers are capped "
                         f"(raise it, e.g. ulimit -l unlimited)", {"soft": soft}))
    if d.get("MemTotal"):
        f.append(Finding("host.memory", "info", f"{d['MemTotal'] >> 20} GiB host memory, "
                                                f"{len(d['numa_nodes'])} NUMA node(s), {d['cpus']} CPUs"))
    return d, f


# ---------------------------------------------------------------- GPU (NVML, read-only)
def _nvml(nvml=None):
    if nvml is not None:
        return nvml, None
    try:
        import pynvml

        pynvml.nvmlInit()
        return pynvml, None
    except Exception as e:  # noqa: BLE001 - no driver / library on this node
        return None, str(e)


def _s(x):
    return x.decode() if isinstance(x, bytes) else x


def gpu_info(nvml=None) -> tuple[dict, list[Finding]]:
    nv, err = _nvml(nvml)
    if nv is None:
        return {"gpus": []}, [Finding("gpu.info", "info", f"NVML unavailable, GPU checks skipped: {err}")]
    f: list[Finding] = []
    n = nv.nvmlDeviceGetCount()
    d = {"driver": _s(nv.nvmlSystemGetDriverVersion()), "gpus": []}
    for i in range(n):
        h = nv.nvmlDeviceGetHandleByIndex(i)
        mem = nv.nvmlDeviceGetMemoryInfo(h)
        g = {"index": i, "name": _s(nv.nvmlDeviceGetName(h)), "memory_total": int(mem.total),
             "memory_used": int(mem.used), "temperature_c": int(nv.nvmlDeviceGetTemperature(h, 0)),
             "sm_clock_mhz": int(nv.nvmlDeviceGetClockInfo(h, 1)),
             "sm_clock_max_mhz": int(nv.nvmlDeviceGetMaxClockInfo(h, 1)),
             "sm_app_clock_mhz": int(nv.nvmlDeviceGetApplicationsClock(h, 1)),
             "power_limit_w": int(nv.nvmlDeviceGetPowerManagementLimit(h)) / 1000.0}
        d["gpus"].append(g)
        if g["sm_app_clock_mhz"] and g["sm_clock_max_mhz"] and g["sm_app_clock_mhz"] < 0.9 * g["sm_clock_max_mhz"]:
            f.append(Finding("gpu.clocks", "warn", f"GPU {i}: application SM clock {g['sm_app_clock_mhz']} MHz is "
                                                   f"below its maximum {g['sm_clock_max_mhz']} MHz (a clock lock is set)",
                             {"gpu": i}))
        if g["temperature_c"] >= 85:
            f.append(Finding("gpu.temperature", "warn", f"GPU {i} at {g['temperature_c']} C", {"gpu": i}))
        if g["memory_used"] > 0.2 * g["memory_total"]:
            f.append(Finding("gpu.memory", "warn", f"GPU {i}: {g['memory_used'] >> 30} GiB already in use",
                             {"gpu": i}))
    names = {g["name"] for g in d["gpus"]}
    if len(names) > 1:
        f.append(Finding("gpu.models", "warn", f"mixed GPU models on one node: {sorted(names)}"))
    f.append(Finding("gpu.info", "info", f"{n} GPU(s) {sorted(names)}, driver {d['driver']}"))
    return d, f


def gpu_topology(nvml=None, max_links: int = B200_NVLINKS) -> tuple[dict, list[Finding]]:
    """Active NVLinks per GPU and the peer-to-peer matrix over NVLink."""
    nv, err = _nvml(nvml)
    if nv is None:
        return {}, [Finding("gpu.topology", "info", f"NVML unavailable, topology skipped: {err}")]
    f: list[Finding] = []
    n = nv.nvmlDeviceGetCount()
    hs = [nv.nvmlDeviceGetHandleByIndex(i) for i in range(n)]
    links = []
    for i, h in enumerate(hs):
        up = 0
        for lk in range(max_links):
            try:
                if nv.nvmlDeviceGetNvLinkState(h, lk):
                    up += 1
            except Exception:  # noqa: BLE001 - link not present
                break
        links.append(up)
        if up < max_links:
            f.append(Finding("gpu.nvlink", "warn", f"GPU {i}: {up} of {max_links} NVLinks active", {"gpu": i}))
    p2p = [[1 if i == j else 0 for j in range(n)] for i in range(n)]
    bad = []
    for i in range(n):
        for j in range(n):
            if i == j:
                continue
            try:
                ok = nv.nvmlDeviceGetP2PStatus(hs[i], hs[j], nv.NVML_P2P_CAPS_INDEX_NVLINK) == nv.NVML_P2P_STATUS_OK
            except Exception:  # noqa: BLE001
                ok = False
            p2p[i][j] = int(ok)
            if not ok:
                bad.append((i, j))
    if bad:
        f.append(Finding("gpu.p2p", "fail", f"{len(bad)} GPU pair(s) without NVLink peer access: {bad[:8]}",
                         {"pairs": bad}))
    elif n > 1:
        f.append(Finding("gpu.p2p", "info", f"all {n * (n - 1)} GPU pairs reach each other over NVLink"))
    return {"nvlinks_active": links, "p2p_nvlink": p2p}, f


# ---------------------------------------------------------------- GPU perf (this repo's kernels)
def _median_outliers(vals: dict, what: str, unit: str, floor: float | None) -> list[Finding]:
    f = []
    if not vals:
        return f
    med = statistics.median(vals.values())
    for k, v in vals.items():
        if v < SLOW_FRAC * med:
            f.append(Finding(what, "warn", f"{k}: {v:.0f} {unit} is below {SLOW_FRAC:.0%} of the node median "
                                           f"{med:.0f}", {"key": str(k), "value": v}))
        if floor is not None and v < floor:
            f.append(Finding(what, "warn", f"{k}: {v:.0f} {unit} is below the B200 floor {floor:.0f}",
                             {"key": str(k), "value": v}))
    return f


def gpu_perf(gemm_n: int = 8192, hbm_bytes: int = 1 << 30, p2p_bytes: int = 1 << 28, iters: int = 20,
             devices: list[int] | None = None) -> tuple[dict, list[Finding]]:
    """Per GPU: bf16 GEMM TFLOP/s through this framework's tcgen05 GEMM
    (``ops.kernels.linear``) and copy bandwidth (read + write bytes over
    ``hbm_bytes``, well above L2); per GPU pair: peer copy GB/s. CUDA events,
    after warm-up."""
    try:
        import torch
    except Exception as e:  # noqa: BLE001
        return {}, [Finding("gpu.perf", "info", f"torch unavailable, perf skipped: {e}")]
    if not torch.cuda.is_available():
        return {}, [Finding("gpu.perf", "info", "no visible GPU, perf skipped")]
    from infera_b200.ops import kernels as K

    devs = devices if devices is not None else list(range(torch.cuda.device_count()))
    gemm, hbm, p2p = {}, {}, {}

    def timed(fn, dev, n):
        with torch.cuda.device(dev):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n):
                fn()
            b.record()
            torch.cuda.synchronize()
            return a.elapsed_time(b) / 1000.0 / n

    for d in devs:
        with torch.cuda.device(d):
            x = torch.randn(gemm_n, gemm_n, device=d, dtype=torch.bfloat16)
            w = torch.randn(gemm_n, gemm_n, device=d, dtype=torch.bfloat16)
            y = torch.empty(gemm_n, gemm_n, device=d, dtype=torch.bfloat16)
            t = timed(lambda: K.linear(x, w, out=y), d, iters)
            gemm[d] = 2 * gemm_n ** 3 / t / 1e12
            del x, w, y
            a = torch.empty(hbm_bytes // 2, device=d, dtype=torch.bfloat16)
            b = torch.empty_like(a)
            t = timed(lambda: b.copy_(a), d, iters)
            hbm[d] = 2 * hbm_bytes / t / 1e9
            del a, b
    for i in devs:
        for j in devs:
            if i == j or not torch.cuda.can_device_access_peer(i, j):
                continue
            src = torch.empty(p2p_bytes, device=i, dtype=torch.uint8)
            dst = torch.empty(p2p_bytes, device=j, dtype=torch.uint8)
            t = timed(lambda: dst.copy_(src, non_blocking=True), i, max(3, iters // 4))
            p2p[f"{i}->{j}"] = p2p_bytes / t / 1e9
            del src, dst
    f = _median_outliers({f"GPU {k}": v for k, v in gemm.items()}, "gpu.gemm", "TFLOP/s", B200_GEMM_MIN_TFLOPS)
    f += _median_outliers({f"GPU {k}": v for k, v in hbm.items()}, "gpu.hbm", "GB/s", B200_HBM_MIN_GBS)
    f += _median_outliers(p2p, "gpu.p2p_copy", "GB/s", B200_P2P_MIN_GBS)
    f.append(Finding("gpu.perf", "info", "bf16 GEMM TFLOP/s " + ", ".join(f"{k}:{v:.0f}" for k, v in gemm.items())
                     + "; copy GB/s " + ", ".join(f"{k}:{v:.0f}" for k, v in hbm.items())))
    return {"gemm_tflops": gemm, "hbm_copy_gbs": hbm, "p2p_copy_gbs": p2p, "gemm_n": gemm_n}, f


# ---------------------------------------------------------------- storage
def nvme_inventory(sys_block: str = "/sys/block") -> list[dict]:
    out = []
    try:
        names = sorted(os.listdir(sys_block))
    except OSError:
        return out
    for n in names:
        if not n.startswith("nvme"):
            continue
        d = {"device": n}
        try:
            with open(os.path.join(sys_block, n, "size")) as fh:
                d["bytes"] = int(fh.read().strip()) * 512
            with open(os.path.join(sys_block, n, "device", "model")) as fh:
                d["model"] = fh.read().strip()
        except OSError:
            pass
        out.append(d)
    return out


def storage(path: str, mib: int = 256, to_gpu: bool = True, sys_block: str = "/sys/block",
            mounts_file: str = "/proc/mounts") -> tuple[dict, list[Finding]]:
    """Where the KV tier directory ``path`` lives, its write / read
    throughput (O_DIRECT where the filesystem takes it), and - with a GPU -
    the staged read into device memory (file -> pinned host -> HBM)."""
    from infera_b200.kvd.storage import classify

    f: list[Finding] = []
    cls = classify(path, mounts_file=mounts_file, sys_block=sys_block)
    d = {"path": path, "kind": cls.kind, "fstype": cls.fstype, "io_mode": cls.io_mode,
         "nvme": nvme_inventory(sys_block)}
    if cls.kind not in ("nvme", "ssd"):
        f.append(Finding("storage.kind", "fail" if cls.kind in ("hdd", "network") else "warn",
                         f"KV tier path {path} is on {cls.kind} ({cls.fstype}), not local NVMe", {"path": path}))
    for w in cls.warnings:
        f.append(Finding("storage.kind", "warn", w))
    os.makedirs(path, exist_ok=True)
    fn = os.path.join(path, f".infera_preflight_{os.getpid()}")
    block = 8 << 20
    n = max(1, mib * (1 << 20) // block)
    import mmap

    buf = mmap.mmap(-1, block)      # page-aligned, as O_DIRECT wants
    buf.write(os.urandom(4096) * (block // 4096))
    flags = os.O_CREAT | os.O_RDWR | (getattr(os, "O_DIRECT", 0) if cls.io_mode == "direct" else 0)
    try:
        try:
            fd = os.open(fn, flags, 0o600)
        except OSError:
            fd = os.open(fn, os.O_CREAT | os.O_RDWR, 0o600)
            d["io_mode"] = "buffered"
        t0 = time.monotonic()
        for i in range(n):
            os.pwrite(fd, buf, i * block)
        os.fsync(fd)
        d["write_gbs"] = n * block / (time.monotonic() - t0) / 1e9
        t0 = time.monotonic()
        for i in range(n):
            os.preadv(fd, [buf], i * block)
        d["read_gbs"] = n * block / (time.monotonic() - t0) / 1e9
        os.close(fd)
        if to_gpu:
            try:
                import torch

                if torch.cuda.is_available():
                    host = torch.empty(block, dtype=torch.uint8, pin_memory=True)
                    dev = torch.empty(block, dtype=torch.uint8, device="cuda")
                    hv = memoryview(host.numpy())
                    fd = os.open(fn, os.O_RDONLY)
                    torch.cuda.synchronize()
                    t0 = time.monotonic()
                    for i in range(n):
                        os.preadv(fd, [hv], i * block)
                        dev.copy_(host, non_blocking=True)
                        torch.cuda.current_stream().synchronize()
                    d["file_to_hbm_gbs"] = n * block / (time.monotonic() - t0) / 1e9
                    os.close(fd)
            except Exception as e:  # noqa: BLE001
                f.append(Finding("storage.to_gpu", "info", f"staged file -> HBM read skipped: {e}"))
    finally:
        try:
            os.unlink(fn)
        except OSError:
            pass
    f.append(Finding("storage.perf", "info", f"{path}: write {d.get('write_gbs', 0):.2f} GB/s, read "
                                             f"{d.get('read_gbs', 0):.2f} GB/s ({d['io_mode']})"
                     + (f", file -> HBM {d['file_to_hbm_gbs']:.2f} GB/s" if "file_to_hbm_gbs" in d else "")))
    return d, f


# ---------------------------------------------------------------- across nodes
def consistency(nodes: dict[str, dict]) -> list[Finding]:
    """Compare node reports: driver, GPU models and GPU count must agree."""
    f = []
    for key, get in (("driver", lambda r: (r.get("gpu") or {}).get("driver")),
                     ("gpu_models", lambda r: tuple(sorted({g["name"] for g in (r.get("gpu") or {}).get("gpus", [])}))),
                     ("gpu_count", lambda r: len((r.get("gpu") or {}).get("gpus", [])))):
        vals = {n: get(r) for n, r in nodes.items()}
        if len({v for v in vals.values()}) > 1:
            f.append(Finding(f"nodes.{key}", "warn", f"{key} differs across nodes: {vals}"))
    return f

"""Build the native parts of infera_b200 in-tree.

* ``infera_b200/lib/libib200_kernels.so`` - every ``csrc/*.cu`` compiled for
  sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), C ABI, no torch
  headers (fast to build, loadable with ctypes, travels with the tree).
* ``infera_b200/lib/ib200_router`` - the native router data plane
  (``native/router/*.cpp``).

Run ``python -m infera_b200.build`` (or ``__graft_entry__.build()``).
Objects are rebuilt only when a source or header is newer than its output.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROUTER_SRC = PKG / "native" / "router"
LIB = PKG / "lib"
OBJ = PKG / "lib" / "obj"

KERNELS_SO = LIB / "libib200_kernels.so"
ROUTER_BIN = LIB / "ib200_router"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _cuda_home() -> Path:
    return Path(_nvcc()).resolve().parent.parent


def _newer(src_files: list[Path], out: Path) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in src_files)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}")


def build_kernels(verbose: bool = False, jobs: int | None = None) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    nvcc = _nvcc()
    objs: list[Path] = []
    todo: list[list[str]] = []
    for src in sources:
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if _newer([src, *headers], obj):
            cmd = [nvcc, *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
                   "-Xcompiler", "-fPIC", "-Xptxas", "-v" if verbose else "-O3",
                   "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
            todo.append(cmd)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(_run, todo))
    if todo or _newer(objs, KERNELS_SO):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(KERNELS_SO), *map(str, objs), "-lcudart"])
    return KERNELS_SO


def xxhash_include() -> Path:
    """Directory holding the reference xxHash header (BSD-2-Clause), which
    the native code includes for XXH3-64: bit-exact with the Python
    ``xxhash`` package by construction. pyarrow vendors a copy."""
    cands = [os.environ.get("XXHASH_INCLUDE")]
    try:
        import pyarrow

        cands.append(os.path.join(pyarrow.get_include(), "arrow", "vendored", "xxhash"))
    except Exception:
        pass
    cands += ["/usr/include", "/usr/local/include"]
    for c in cands:
        if c and (Path(c) / "xxhash.h").exists():
            return Path(c)
    raise RuntimeError("xxhash.h not found (set XXHASH_INCLUDE)")


SANITIZERS = {
    # name: compile / link flags (race and memory checking of the host code;
    # the GPU-side sanitizer is not available on the GPU machines)
    "asan": ["-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"],
    "tsan": ["-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=thread"],
}


def build_router(sanitize: str | None = None) -> Path | None:
    """The native router; ``sanitize`` ("asan" = AddressSanitizer +
    UndefinedBehaviorSanitizer, "tsan" = ThreadSanitizer) builds
    ``ib200_router_<name>`` next to the release binary."""
    sources = sorted(ROUTER_SRC.glob("*.cpp")) if ROUTER_SRC.exists() else []
    if not sources:
        return None
    headers = sorted(ROUTER_SRC.glob("*.h"))
    flags = ["-O2"] if sanitize is None else SANITIZERS[sanitize]
    out_bin = ROUTER_BIN if sanitize is None else LIB / f"ib200_router_{sanitize}"
    tag = "router_" if sanitize is None else f"router_{sanitize}_"
    if _newer([*sources, *headers], out_bin):
        LIB.mkdir(parents=True, exist_ok=True)
        objs = []
        todo = []
        for src in sources:
            obj = OBJ / (tag + src.stem + ".o")
            objs.append(obj)
            if _newer([src, *headers], obj):
                todo.append(["g++", *flags, "-std=c++17", "-Wall", "-I", str(ROUTER_SRC), "-I", str(xxhash_include()),
                             "-c", str(src), "-o", str(obj)])
        OBJ.mkdir(parents=True, exist_ok=True)
        if todo:
            with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
                list(ex.map(_run, todo))
        link = [] if sanitize is None else [f for f in flags if f.startswith("-fsanitize")]
        _run(["g++", *link, "-o", str(out_bin), *map(str, objs), "-lpthread", "-lssl", "-lcrypto"])
    return out_bin


def build_all(verbose: bool = False) -> dict[str, str | None]:
    out = {"kernels": str(build_kernels(verbose=verbose))}
    rb = build_router()
    out["router"] = str(rb) if rb else None
    return out


if __name__ == "__main__":
    res = build_all(verbose="-v" in sys.argv)
    for k, v in res.items():
        print(f"{k}: {v}")

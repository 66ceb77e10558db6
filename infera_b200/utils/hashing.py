"""Chained block hashing shared by the engine's prefix cache and the router.

``h_i = XXH3_64(h_{i-1} as u64 LE || block tokens as u32 LE)``, seed 0,
``h_{-1} = 0``; a trailing partial block is dropped. Bit-exact with the
reference router (``infera/router/kv_event/hasher.py:20-42``) because the
wire-visible hashes must agree across the fleet.

The native runtime library (C++ XXH3) is used when it is built; the Python
``xxhash`` package is the fallback and the oracle.
"""

from __future__ import annotations

import ctypes

import numpy as np
import xxhash

ROUTER_SEED = 0


def hash_chunk(parent: int, token_ids) -> int:
    buf = int(parent).to_bytes(8, "little", signed=False) + np.asarray(token_ids, dtype=np.uint32).tobytes()
    return xxhash.xxh3_64_intdigest(buf)


def _chain_py(token_ids, block_size: int, parent: int) -> list[int]:
    arr = np.asarray(token_ids, dtype=np.uint32)
    n_full = len(arr) // block_size
    if n_full == 0:
        return []
    raw = arr[: n_full * block_size].tobytes()
    step = 4 * block_size
    out = []
    h = parent
    f = xxhash.xxh3_64_intdigest
    for i in range(n_full):
        h = f(h.to_bytes(8, "little") + raw[i * step:(i + 1) * step])
        out.append(h)
    return out


_native_fn = None
_native_checked = False


def _native():
    global _native_fn, _native_checked
    if not _native_checked:
        _native_checked = True
        try:
            from infera_b200.ops._native import runtime

            lib = runtime()
            if lib is not None and hasattr(lib, "ib_chain_hashes"):
                fn = lib.ib_chain_hashes
                fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p]
                fn.restype = ctypes.c_longlong
                _native_fn = fn
        except Exception:  # pragma: no cover - library optional on CPU
            _native_fn = None
    return _native_fn


def chain_hashes(token_ids, block_size: int, parent: int = ROUTER_SEED) -> list[int]:
    """Chained hashes of every full block of ``token_ids``."""
    if block_size <= 0:
        return []
    fn = _native()
    if fn is None:
        return _chain_py(token_ids, block_size, parent)
    arr = np.ascontiguousarray(np.asarray(token_ids, dtype=np.uint32))
    n_full = len(arr) // block_size
    if n_full == 0:
        return []
    out = np.empty(n_full, dtype=np.uint64)
    fn(arr.ctypes.data, len(arr), block_size, parent, out.ctypes.data)
    return [int(x) for x in out]


def hash_request(token_ids, block_size: int) -> list[int]:
    """Router-side name of :func:`chain_hashes` from seed 0."""
    return chain_hashes(token_ids, block_size, ROUTER_SEED)

"""Loader for the in-tree native libraries.

``libib200_kernels.so`` holds every sm_100a CUDA kernel behind a C ABI,
built in-tree by :mod:`infera_b200.build` and loaded with :mod:`ctypes`
(the native router is a separate executable).

On a machine with a GPU a missing kernel library is an error, never a silent
fallback: :func:`kernels` raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_DIR = Path(__file__).resolve().parent.parent / "lib"
_lock = threading.Lock()
_kernels: ctypes.CDLL | None = None

c_int = ctypes.c_int
c_ll = ctypes.c_longlong
c_float = ctypes.c_float
c_uint = ctypes.c_uint
c_vp = ctypes.c_void_p
c_ip = ctypes.c_void_p  # int* passed as raw address


def kernel_lib_path() -> Path:
    return _LIB_DIR / "libib200_kernels.so"


def _declare_kernels(lib: ctypes.CDLL) -> None:
    sig = {
        "ib_gemm_bf16": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_int, c_vp,
                         c_vp],
        "ib_gemm_bf16_plan": [c_int, c_int, c_int, c_int, c_int, c_vp],
        "ib_rmsnorm": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float, c_vp],
        "ib_add_rmsnorm": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_float, c_vp],
        "ib_add_rmsnorm_ws": [c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float, c_vp],
        "ib_rope_kvwrite_ws": [c_vp, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp,
                               c_int, c_ll, c_int, c_vp, c_vp],
        "ib_gemm_bf16_deferred": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp,
                                  c_vp],
        "ib_rope_kvwrite": [c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp, c_int, c_ll,
                            c_int, c_vp, c_vp],
        "ib_embed": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp],
        "ib_sample": [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp],
        "ib_gather_rows": [c_vp, c_vp, c_vp, c_int, c_int, c_vp],
        "ib_attn_decode": [c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_float,
                           c_vp, c_vp, c_vp, c_int, c_vp],
        "ib_attn_prefill": [c_vp, c_int, c_int, c_vp, c_vp, c_ll, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_int,
                            c_int, c_int, c_float, c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_int, c_vp],
        "ib_attn_prefill_ext": [c_vp, c_int, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int,
                                c_int, c_vp, c_int, c_int, c_ll, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_int,
                                c_int, c_int, c_float, c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_vp],
        "ib_scatter_i32": [c_vp, c_vp, c_vp, c_int, c_vp],
        "ib_kv_page_copy": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_ll, c_int, c_int, c_int, c_int, c_vp],
        "ib_attn_decode_tc": [c_vp, c_int, c_vp, c_vp, c_ll, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int,
                              c_float, c_vp, c_vp, c_vp, c_int, c_vp, c_vp],
        "ib_attn_decode_tc_ex": [c_vp, c_int, c_vp, c_vp, c_ll, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int,
                                 c_float, c_vp, c_vp, c_vp, c_int, c_vp, c_int, c_int, c_vp],
        "ib_gemm_bf16_push": [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp,
                              c_vp, c_vp],
        "ib_ar_add_rmsnorm": [c_vp, c_ll, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp, c_float, c_vp,
                              c_vp, c_vp],
        "ib_sym_alloc": [ctypes.c_size_t, c_vp],
        "ib_sym_free": [c_vp],
        "ib_ipc_handle": [c_vp, c_vp],
        "ib_ipc_open": [c_vp, c_vp],
        "ib_ipc_close": [c_vp],
        "ib_can_access_peer": [c_int, c_int],
        "ib_enable_peer_access": [c_int],
        "ib_moe_topk": [c_vp, c_int, c_int, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_vp, c_vp,
                        c_vp],
        "ib_moe_permute": [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_moe_tiles": [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp],
        "ib_moe_combine": [c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_int, c_vp],
        "ib_ep_offsets": [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp],
        "ib_ep_dispatch": [c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_ep_return": [c_vp, c_int, c_int, c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_ep_wait": [c_vp, ctypes.c_uint, c_vp, c_vp],
        "ib_ep_wait_for": [c_vp, ctypes.c_uint, c_vp, ctypes.c_ulonglong, c_vp],
        "ib_gemm_grouped": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp,
                            c_int, c_int, c_vp, c_vp],
        "ib_kv_push_pages": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_ll, c_ll, c_int, c_int, c_int,
                             c_vp],
        "ib_gemm_fp8": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp,
                        c_int, c_vp, c_vp],
        "ib_gemm_fp8_push": [c_vp, c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp,
                             c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_gemm_fp8_grouped": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int,
                                c_int, c_int, c_vp, c_vp, c_int, c_int, c_vp, c_vp],
        "ib_gemm_fp8_plan": [c_int, c_int, c_int, c_int, c_int, c_vp],
        "ib_quant_fp8_act": [c_vp, c_int, c_int, c_int, c_vp, c_int, c_vp, c_int, c_vp],
        "ib_gemm_bf16_push_rs": [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp,
                                 c_vp, c_vp, c_vp],
        "ib_gemm_fp8_push_rs": [c_vp, c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_ar_add_rmsnorm_rs": [c_vp, c_ll, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_float,
                                 c_vp, c_vp, c_vp, c_vp],
        "ib_tp_wait": [c_vp, ctypes.c_uint, c_vp, c_vp],
        "ib_tp_wait_for": [c_vp, ctypes.c_uint, c_vp, ctypes.c_ulonglong, c_vp],
        "ib_tp_wait_next": [c_vp, c_vp, ctypes.c_uint, c_vp, c_vp],
        "ib_mla_decode": [c_vp, c_int, c_int, c_vp, c_ll, c_vp, c_vp, c_vp, c_int, c_int, c_float, c_vp, c_vp, c_vp,
                          c_vp, c_vp],
        "ib_mla_key_tile": [],
        "ib_mla_set_trace": [c_vp],
        "ib_ep_row_map": [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_int, c_vp, c_vp],
        "ib_gemm_grouped_push": [c_vp, c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                 c_vp, c_vp, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_gemm_grouped_wait": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int,
                                 c_int, c_int, c_vp, c_vp, c_int, c_int, c_vp, c_uint, c_vp, c_vp],
        "ib_gemm_grouped_wait_for": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int,
                                     c_int, c_int, c_vp, c_vp, c_int, c_int, c_vp, c_uint, ctypes.c_ulonglong, c_vp,
                                     c_vp],
        "ib_ep_dispatch_q": [c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_int,
                             c_vp, c_vp, c_vp],
        "ib_ep_dispatch_ex": [c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_ep_dispatch_q_ex": [c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_int,
                                c_vp, c_vp, c_vp, c_vp, c_vp],
        "ib_gemm_grouped_wait_ex": [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int,
                                    c_int, c_int, c_vp, c_vp, c_int, c_int, c_vp, c_uint, c_int, ctypes.c_ulonglong,
                                    c_vp, c_vp],
        "ib_gemm_set_trace": [c_vp],
        "ib_gemm_set_tile_counters": [c_vp, c_int],
        "ib_gemm_fused_reduce": [],
        "ib_attn_prefill_set_trace": [c_vp],
        "ib_mla_rope_kvwrite": [c_vp, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_float, c_vp, c_vp],
    }
    for name, args in sig.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.argtypes = args
        fn.restype = None if name in ("ib_gemm_bf16_plan", "ib_gemm_fp8_plan", "ib_mla_set_trace",
                                        "ib_gemm_set_trace", "ib_attn_prefill_set_trace",
                                        "ib_gemm_set_tile_counters") else c_int


def kernels() -> ctypes.CDLL:
    """The CUDA kernel library; raises if it was not built."""
    global _kernels
    if _kernels is None:
        with _lock:
            if _kernels is None:
                path = kernel_lib_path()
                if not path.exists():
                    raise RuntimeError(
                        f"{path} is missing: build it with `python -m infera_b200.build` "
                        "(the CUDA path has no fallback)")
                lib = ctypes.CDLL(str(path), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
                _declare_kernels(lib)
                _kernels = lib
    return _kernels


# INFERA_SYNC_CHECK=1: synchronise after every launch, so a device fault is
# reported against the kernel that caused it (slow; for diagnosis)
_SYNC_CHECK = os.environ.get("INFERA_SYNC_CHECK", "") == "1"


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with code {rc}")
    if _SYNC_CHECK:
        import torch

        if torch.cuda.is_available():
            try:
                torch.cuda.synchronize()
            except RuntimeError as e:
                raise RuntimeError(f"{what}: device error after this launch: {e}") from e
            if status_probe is not None:
                st = status_probe()
                if st and st.get("code"):
                    raise RuntimeError(f"{what}: kernel status after this launch: {st}")


# set by the kernel wrappers: reads the current device's status word and
# details (used by INFERA_SYNC_CHECK)
status_probe = None

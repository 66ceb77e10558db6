"""The allocation-free decode-attention entry point, called through its
exported C symbol.

Some callers of this library cannot allocate device memory themselves: a
plugin inside a host framework that owns all GPU memory through its own
capped pool, or a latency-critical path where cudaMalloc would synchronise
the device. ``ib_attn_decode_noalloc`` serves them: they pass inputs and
the output only, and the split-KV partials live in a fixed array inside the
library. This test checks that it matches the regular entry point (which
takes caller-provided scratch) on two calls in a row - the second call
reuses the array the first one left behind - and that an oversized call is
rejected without launching anything.

The file name makes pytest collect it last.
"""

import ctypes
import math

import pytest
import torch

from infera_b200.ops import _native
from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu

TOO_BIG = -3


def _fn():
    _native.kernels()  # loads the library (and fails loudly if it is missing)
    lib = ctypes.CDLL(str(_native.kernel_lib_path()))
    fn = lib.ib_attn_decode_noalloc
    c_int, c_vp = ctypes.c_int, ctypes.c_void_p
    fn.argtypes = [c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, ctypes.c_float,
                   c_vp, c_int, c_vp]
    fn.restype = c_int
    lib.ib_attn_decode_noalloc_max_rows.restype = c_int
    return fn, lib.ib_attn_decode_noalloc_max_rows()


def _case(lens, seed, hq=32, hkv=8, D=128):
    g = torch.Generator().manual_seed(seed)
    pages = sum((n + 15) // 16 for n in lens) + 2
    perm = torch.randperm(pages, generator=g)
    width = max((n + 15) // 16 for n in lens)
    bt = torch.zeros(len(lens), width, dtype=torch.int32)
    k = 0
    for i, n in enumerate(lens):
        for j in range((n + 15) // 16):
            bt[i, j] = perm[k]
            k += 1
    kc = torch.randn(pages * 16, hkv * D, generator=g).to(torch.bfloat16).cuda()
    vc = torch.randn(pages * 16, hkv * D, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(len(lens), (hq + 2 * hkv) * D, generator=g).to(torch.bfloat16).cuda()
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32).cuda()


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-6))


def test_noalloc_matches_allocating_entry_point_twice():
    fn, max_rows = _fn()
    hq, hkv = 32, 8
    scale = 1 / math.sqrt(128)
    for call, (lens, splits) in enumerate([([700, 33, 2048, 5], 8), ([4000, 1, 129], 16)]):
        assert len(lens) * hq * splits <= max_rows
        q, kc, vc, bt, sl = _case(lens, seed=call)
        want = K.attn_decode(q, kc, vc, bt, sl, hq, hkv, scale, splits=splits)
        got = torch.full_like(want, float("nan"))
        rc = fn(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), None, sl.data_ptr(),
                bt.stride(0), len(lens), hq, hkv, splits, scale, got.data_ptr(), got.stride(0),
                torch.cuda.current_stream().cuda_stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert _rel_err(got, want) < 2e-2, call


def test_noalloc_rejects_oversized_batches():
    fn, max_rows = _fn()
    hq, hkv = 32, 8
    lens = [64] * 8
    splits = max_rows // (len(lens) * hq) + 1
    q, kc, vc, bt, sl = _case(lens, seed=3)
    out = torch.zeros(len(lens), hq * 128, dtype=torch.bfloat16, device="cuda")
    rc = fn(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), None, sl.data_ptr(),
            bt.stride(0), len(lens), hq, hkv, splits, 1.0, out.data_ptr(), out.stride(0),
            torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_BIG
    torch.cuda.synchronize()
    assert float(out.float().abs().sum()) == 0.0

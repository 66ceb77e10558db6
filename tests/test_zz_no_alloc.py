"""The allocation-free decode-attention entry point, called through its
exported C symbol.

Some callers of this library cannot allocate device memory themselves: a
plugin inside a host framework that owns all GPU memory through its own
capped pool, or a latency-critical path where cudaMalloc would synchronise
the device. ``ib_attn_decode_noalloc`` serves them: they pass inputs and
the output only, and the split-KV partials live in a fixed array inside the
library. These tests check it against an fp32 CPU restatement of the
attention and against the regular entry point (which takes caller-provided
scratch), on two calls in a row - the second call reuses the array the
first one left behind - for every supported GQA group size and for the
single-split path that needs no scratch; that device memory stays exactly
as free as before the calls; and that an oversized call is rejected without
launching anything.

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
TOL = 2e-2


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


def _oracle(q, kc, vc, bt, sl, hq, hkv, scale):
    """fp32 attention on the CPU (the same restatement the kernels' other
    numerics tests use)."""
    return K.attn_decode(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), hq, hkv, scale).float()


def _rel_err(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-6))


def _call(fn, q, kc, vc, bt, sl, hq, hkv, splits, scale, out):
    return fn(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), None, sl.data_ptr(),
              bt.stride(0), sl.shape[0], hq, hkv, splits, scale, out.data_ptr(), out.stride(0),
              torch.cuda.current_stream().cuda_stream)


# (query heads, KV heads, sequence lengths, splits): GQA groups 1, 2, 4, 8,
# and splits == 1, the path that uses no scratch and has no size limit
CASES = [
    (32, 8, [700, 33, 2048, 5], 8),
    (32, 8, [4000, 1, 129], 16),
    (8, 8, [300, 1500], 4),
    (16, 8, [999, 64, 17], 1),
    (64, 8, [2500, 40], 2),
]


@pytest.mark.parametrize("hq,hkv,lens,splits", CASES)
def test_noalloc_matches_oracle_and_allocating_entry_point_twice(hq, hkv, lens, splits):
    fn, max_rows = _fn()
    assert len(lens) * hq * splits <= max_rows
    scale = 1 / math.sqrt(128)
    for call in range(2):     # the second call finds the first call's partials in the shared array
        q, kc, vc, bt, sl = _case(lens, seed=100 * hq + 10 * splits + call, hq=hq, hkv=hkv)
        want = _oracle(q, kc, vc, bt, sl, hq, hkv, scale)
        alloc = K.attn_decode(q, kc, vc, bt, sl, hq, hkv, scale, splits=splits, impl="simt")
        got = torch.full_like(alloc, float("nan"))
        rc = _call(fn, q, kc, vc, bt, sl, hq, hkv, splits, scale, got)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert _rel_err(got, want) < TOL, (call, _rel_err(got, want))
        assert _rel_err(got, alloc) < TOL, (call, _rel_err(got, alloc))
    assert K.scratch(q.device).read_status() == 0


def test_noalloc_calls_take_no_device_memory():
    """After the first call on the device (which looks up the array's
    address; the array itself is part of the library's device image), the
    calls leave device memory exactly as free as they found it."""
    fn, _ = _fn()
    hq, hkv, splits = 32, 8, 8
    scale = 1 / math.sqrt(128)
    q, kc, vc, bt, sl = _case([1200, 77, 3000], seed=7)
    outs = [torch.zeros(3, hq * 128, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    assert _call(fn, q, kc, vc, bt, sl, hq, hkv, splits, scale, outs[0]) == 0   # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for o in outs[1:]:
        assert _call(fn, q, kc, vc, bt, sl, hq, hkv, splits, scale, o) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.equal(outs[1], outs[2]) and torch.equal(outs[0], outs[1])


def test_noalloc_rejects_oversized_batches():
    fn, max_rows = _fn()
    hq, hkv = 32, 8
    lens = [64] * 8
    splits = max_rows // (len(lens) * hq) + 1
    q, kc, vc, bt, sl = _case(lens, seed=3)
    out = torch.zeros(len(lens), hq * 128, dtype=torch.bfloat16, device="cuda")
    rc = _call(fn, q, kc, vc, bt, sl, hq, hkv, splits, 1.0, out)
    assert rc == TOO_BIG
    torch.cuda.synchronize()
    assert float(out.float().abs().sum()) == 0.0

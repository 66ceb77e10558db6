"""Device-side waits that run out, on one GPU, with the context left usable.

The fused NVLink paths wait on flags that other GPUs set (the TP owners'
arrival counter, the EP dispatch's arrival counter, which the up
projection's TMA producer waits on itself). Every such wait is bounded; on
expiry the kernel writes a status code, releases whatever it holds (the
grouped GEMM drains its copies and frees its TMEM) and returns. Here each
wait is pointed at a flag that nothing sets, with a 10 ms limit: the status
must show the timeout within well under a second, and the same kernels then
run to a clean, correct result on the same GPU.
"""

import ctypes
import time

import pytest
import torch

from infera_b200.ops import _native
from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu

TIMEOUT_PEER = 5          # kStatusTimeoutPeer (grouped GEMM arrival wait)
TIMEOUT_TP = 0x4101       # tensor-parallel owner-arrival wait
TIMEOUT_EP = 0x4201       # expert-parallel dispatch-arrival wait
LIMIT_NS = 10_000_000     # 10 ms


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _grouped_wait(x, w, off, out, flag, target, status):
    R, Kd = x.shape
    E, N, _ = w.shape
    bn = K.grouped_bn(R, E)
    tab, num, cap = K.grouped_tiles(off, E, N, bn, R)
    rc = _native.kernels().ib_gemm_grouped_wait_for(
        x.data_ptr(), None, 0, w.data_ptr(), None, out.data_ptr(), R, N, Kd, E, x.stride(0), w.stride(1),
        out.stride(0), 0, tab.data_ptr(), num.data_ptr(), bn, cap, flag.data_ptr(), target, LIMIT_NS,
        status.data_ptr(), _stream())
    _native.check(rc, "ib_gemm_grouped_wait_for")


def _timed(fn):
    torch.cuda.synchronize()
    t0 = time.monotonic()
    fn()
    torch.cuda.synchronize()
    return time.monotonic() - t0


def test_flag_waits_time_out_and_report():
    lib = _native.kernels()
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for name, code in (("ib_tp_wait_for", TIMEOUT_TP), ("ib_ep_wait_for", TIMEOUT_EP)):
        fn = getattr(lib, name)
        status.zero_()
        dt = _timed(lambda: _native.check(fn(flag.data_ptr(), 1, status.data_ptr(), LIMIT_NS, _stream()), name))
        assert int(status.item()) == code, name
        assert dt < 1.0, (name, dt)
        # the same wait on a flag that has arrived returns at once, status clean
        status.zero_()
        flag[0] = 1
        _native.check(fn(flag.data_ptr(), 1, status.data_ptr(), LIMIT_NS, _stream()), name)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, name
        flag.zero_()


def test_grouped_gemm_arrival_wait_times_out_then_runs_clean():
    g = torch.Generator().manual_seed(5)
    E, N, Kd = 4, 256, 512
    counts = [40, 0, 77, 11]
    off = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32)
    R = int(off[-1])
    x = (torch.randn(R, Kd, generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(E, N, Kd, generator=g) * 0.05).to(torch.bfloat16)
    want = K.gemm_grouped(x, w, off)                       # fp32 CPU oracle
    xd, wd, offd = x.cuda(), w.cuda(), off.cuda()
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros(R, N, dtype=torch.bfloat16, device="cuda")
    # nobody sets the flag: the producer gives up after 10 ms, the CTA's other
    # roles are released, TMEM is freed, the launch completes
    dt = _timed(lambda: _grouped_wait(xd, wd, offd, out, flag, 1, status))
    assert int(status.item()) == TIMEOUT_PEER
    assert dt < 1.0, dt
    # the same kernel on the same GPU, flag arrived: correct result, clean status
    status.zero_()
    flag[0] = 1
    _grouped_wait(xd, wd, offd, out, flag, 1, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    err = float((out.float().cpu() - want.float()).norm() / want.float().norm())
    assert err < 1e-2, err
    # and an unrelated kernel afterwards
    y = K.linear(xd, wd[0])
    torch.cuda.synchronize()
    ref = x.float() @ w[0].float().t()
    assert float((y.float().cpu() - ref).norm() / ref.norm()) < 1e-2

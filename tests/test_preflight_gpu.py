"""Preflight GPU probes on a real B200: NVML reads (query calls only) and the
GEMM / copy measurements through this framework's kernels."""

import pytest

from infera_b200.preflight import checks

pytestmark = pytest.mark.gpu


def test_gpu_info_and_perf_on_b200():
    d, f = checks.gpu_info()
    assert d["gpus"] and "B200" in d["gpus"][0]["name"]
    p, pf = checks.gpu_perf(gemm_n=4096, hbm_bytes=1 << 29, iters=10, devices=[0])
    assert p["gemm_tflops"][0] > 300 and p["hbm_copy_gbs"][0] > 2000, p

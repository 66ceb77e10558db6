"""Expert-parallel MoE on GPUs against the single-device fp32-accumulated
layer: the NCCL all-to-all path and the fused NVLink peer-store dispatch /
return path (``ib_ep_*``). World 1 runs the fused kernels against its own
buffers on one GPU (dispatch, bounded arrival wait, grouped GEMMs, return)."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(nproc: int, port: int, *extra: str) -> dict:
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(nproc), "--master-addr", "127.0.0.1", "--master-port", str(port), "-m",
           "infera_b200.bench.ep_check", "--tokens", "40", "--hidden", "1024", "--ffn", "512", "--experts", "32",
           "--top-k", "4", "--iters", "5", *extra]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    res = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    assert res["max_rel_err"] < 2e-2, res
    assert all(rk.get("status", 0) == 0 for rk in res["ranks"]), res
    return res


def test_ep_fused_single_rank():
    res = _run(1, 29771, "--fused")
    assert res["ranks"][0]["fused"]


def test_ep_fused_single_rank_fp8():
    """fp8 experts: the sender quantises, ib_ep_dispatch_q moves e4m3 rows
    with their scale columns, and the up projection waits for them inside
    its own producer (ib_gemm_grouped_wait)."""
    res = _run(1, 29774, "--fused", "--fp8")
    assert res["ranks"][0]["fused"]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_nccl_two_ranks():
    _run(2, 29772)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_fused_two_ranks():
    res = _run(2, 29773, "--fused")
    assert all(rk["fused"] for rk in res["ranks"])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_fused_two_ranks_fp8():
    res = _run(2, 29778, "--fused", "--fp8")
    assert all(rk["fused"] for rk in res["ranks"])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [False, True])
def test_dp_attention_ep_two_gpus(fused):
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(29775 + int(fused)), "-m",
           "infera_b200.bench.dp_check", "--model", "tiny-mla-gpu", "--prompts", "5"] + (["--fused"] if fused else [])
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=330)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    res = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    assert res["agreement"] >= 0.9, res


def test_dp_attention_ep_one_gpu_fused_layers_share_buffers():
    """World 1, fused path, two MoE layers: every EP layer of the process
    uses one set of symmetric buffers and one round counter (full-size
    DeepSeek-V3 shards cannot afford a set per layer)."""
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "1", "--master-addr", "127.0.0.1", "--master-port", "29779", "-m",
           "infera_b200.bench.dp_check", "--model", "tiny-mla-gpu", "--prompts", "4", "--fused"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=330)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    res = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    assert res["agreement"] >= 0.9, res

"""Tensor-parallel fused GEMM + all-reduce + add + RMSNorm (NVLink peer
stores) against a single-GPU fp32 computation of the whole problem, and
against the NCCL baseline path."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_fused_allreduce_single_rank():
    from infera_b200.bench.tp_comm_bench import main

    # world 1 exercises the push / arrival / consume bookkeeping on one GPU
    main(["--rows", "1,64,200", "--hidden", "4096", "--k-total", "2048", "--check-only"])


def test_two_shot_single_rank():
    from infera_b200.bench.tp_comm_bench import main

    # reduce-scatter epilogue + owner reduce / broadcast + wait, on one GPU
    main(["--rows", "64,300,1024", "--hidden", "4096", "--k-total", "2048", "--check-only",
          "--one-shot-rows", "128"])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_shot_two_ranks():
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29613", "-m",
           "infera_b200.bench.tp_comm_bench", "--rows", "256,700,2048", "--one-shot-rows", "256", "--check-only"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    assert r.returncode == 0, r.stdout.decode()[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_allreduce_two_ranks():
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29611", "-m",
           "infera_b200.bench.tp_comm_bench", "--rows", "1,64,256", "--check-only"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    assert r.returncode == 0, r.stdout.decode()[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_engine_matches_single_gpu():
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29612", "-m",
           "infera_b200.bench.tp_engine_check", "--model", "llama-3.1-8b", "--batch", "8", "--decode-steps", "24"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=330)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    line = [x for x in out.splitlines() if x.startswith("{")][-1]
    import json

    res = json.loads(line)
    assert res["status"] == 0
    # every divergence from the single-GPU model is at a rounding tie
    assert res["greedy_agreement"] >= 0.9 or res["max_rel_gap_at_divergence"] < 0.01, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_lm_head_fused_gather_two_ranks():
    """The vocab-parallel LM head whose epilogue stores every rank's column
    block into every rank's logits, against the fp32 product of the whole
    weight and against GEMM + NCCL all-gather."""
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29614", "-m",
           "infera_b200.bench.tp_comm_bench", "--lm-head", "128256", "--hidden", "4096", "--rows", "1,37,128",
           "--check-only"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    assert r.returncode == 0, r.stdout.decode()[-3000:]

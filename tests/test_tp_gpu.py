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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_worker_serves_over_http():
    """``python -m infera_b200.engine.worker --tp-size 2``: the worker launches
    its two engine-core ranks with torch.distributed.run and serves the
    OpenAI API; greedy completions come back."""
    import json
    import time

    import httpx

    from infera_b200.common.net import free_tcp_port

    port = free_tcp_port()
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    p = subprocess.Popen([sys.executable, "-m", "infera_b200.engine.worker", "--model", "llama-3.1-8b",
                          "--tp-size", "2", "--port", str(port), "--max-num-seqs", "16", "--log-level", "warning"],
                         env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, start_new_session=True)
    url = f"http://127.0.0.1:{port}"
    try:
        t0 = time.time()
        while time.time() - t0 < 400:
            try:
                if httpx.get(url + "/health", timeout=2).status_code == 200:
                    break
            except httpx.HTTPError:
                pass
            if p.poll() is not None:
                raise AssertionError(p.stdout.read().decode()[-3000:])
            time.sleep(1)
        outs = []
        for prompt in ([1, 2, 3, 4, 5, 6, 7, 8], list(range(100, 400))):
            r = httpx.post(url + "/v1/completions", json={"model": "llama-3.1-8b", "prompt": prompt, "max_tokens": 8,
                                                          "ignore_eos": True, "return_token_ids": True}, timeout=120)
            assert r.status_code == 200, r.text
            outs.append(r.json()["choices"][0])
        assert all(len(o.get("token_ids") or []) == 8 for o in outs), json.dumps(outs)[:500]
    finally:
        import signal as _signal

        os.killpg(p.pid, _signal.SIGTERM)
        try:
            p.wait(timeout=60)
        except subprocess.TimeoutExpired:
            os.killpg(p.pid, _signal.SIGKILL)

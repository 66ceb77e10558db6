"""Data-parallel attention ranks served over HTTP (CPU, 2 gloo ranks):
two engine cores started by torch.distributed.run share the MoE experts
(EP over gloo) and step in lockstep; one HTTP worker per rank, registered
with its dp_rank, serves completions; a request on one rank completes while
the other rank idles, and both ranks' answers match single-engine greedy
decoding of the same prompts."""

import asyncio
import json
import os
import subprocess
import sys
import time

import httpx

from infera_b200.common.net import free_tcp_port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _wait(url, timeout=120):
    t0 = time.time()
    while time.time() - t0 < timeout:
        try:
            if httpx.get(url, timeout=1).status_code == 200:
                return True
        except httpx.HTTPError:
            pass
        time.sleep(0.2)
    return False


def test_dp_attention_serving_two_ranks_cpu(tmp_path):
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams

    env = dict(os.environ, PYTHONPATH=ROOT)
    tag = f"ib200-dp-{os.getpid()}"
    in_t, out_t = f"ipc:///tmp/{tag}-in-{{rank}}", f"ipc:///tmp/{tag}-out-{{rank}}"
    core = subprocess.Popen([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                             "--master-addr", "127.0.0.1", "--master-port", str(free_tcp_port()), "-m",
                             "infera_b200.engine.core_ipc", "--in", in_t, "--out", out_t, "--model", "tiny-moe",
                             "--device", "cpu", "--num-pages", "64", "--max-batched-tokens", "64",
                             "--max-num-seqs", "4", "--dp-attention-size", "2"],
                            env=env, cwd=ROOT, stdout=open(tmp_path / "core.log", "w"), stderr=subprocess.STDOUT,
                            start_new_session=True)
    workers, ports = [], []
    try:
        for r in range(2):
            port = free_tcp_port()
            ports.append(port)
            workers.append(subprocess.Popen(
                [sys.executable, "-m", "infera_b200.engine.worker", "--model", "tiny-moe", "--port", str(port),
                 "--attach-core", f"{in_t.format(rank=r)},{out_t.format(rank=r)}", "--dp-rank", str(r),
                 "--dp-size", "2", "--log-level", "warning"],
                env=env, cwd=ROOT, stdout=open(tmp_path / f"w{r}.log", "w"), stderr=subprocess.STDOUT,
                start_new_session=True))
        for port in ports:
            assert _wait(f"http://127.0.0.1:{port}/health"), (tmp_path / "core.log").read_text()[-3000:]
        prompts = [[5, 17, 99, 3, 250, 7], [300, 1, 42, 42, 8]]

        async def go():
            async with httpx.AsyncClient(timeout=120) as c:
                # rank 1 alone first (rank 0 idles in step), then both at once
                r1 = await c.post(f"http://127.0.0.1:{ports[1]}/v1/completions",
                                  json={"model": "tiny-moe", "prompt": prompts[1], "max_tokens": 4,
                                        "ignore_eos": True, "return_token_ids": True})
                both = await asyncio.gather(*(c.post(f"http://127.0.0.1:{ports[i]}/v1/completions",
                                                     json={"model": "tiny-moe", "prompt": prompts[i],
                                                           "max_tokens": 4, "ignore_eos": True,
                                                           "return_token_ids": True}) for i in range(2)))
                return [r1] + list(both)

        res = asyncio.run(go())
        ids = [r.json()["choices"][0]["token_ids"] for r in res]
        ref = LLMEngine(EngineConfig(model="tiny-moe", use_cuda_graphs=False, num_pages=64),
                        device="cpu").generate(prompts, SamplingParams(max_tokens=4, ignore_eos=True))
        assert ids[0] == ref[1] and ids[1] == ref[0] and ids[2] == ref[1], (ids, ref)
    finally:
        for w in workers:
            w.terminate()
        for w in workers:
            try:
                w.wait(timeout=20)
            except subprocess.TimeoutExpired:
                w.kill()
        core.terminate()
        try:
            core.wait(timeout=30)
        except subprocess.TimeoutExpired:
            os.killpg(core.pid, 9)

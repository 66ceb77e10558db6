"""The DP-attention + EP serving replay on two gloo ranks: the ranks vote
each iteration (work, end of window), step in lockstep with dummy forwards
on the idle rank, and rank 0 reports the cohort over both ranks."""

import json
import os
import subprocess
import sys

from infera_b200.common.net import free_tcp_port


def test_ep_serve_two_gloo_ranks():
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=repo)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(free_tcp_port()), "-m", "infera_b200.bench.ep_serve", "--cpu",
           "--model", "tiny-moe", "--trace", "tiny", "--rate", "4", "--warmup", "1", "--duration", "3", "--tail",
           "4", "--max-batched-tokens", "64", "--max-num-seqs", "4"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=240, env=env, cwd=repo)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    assert d["parallelism"] == "EP2 + DP-attention2"
    assert d["arrived"] > 0 and d["completed"] == d["arrived"]
    assert len(d["idle_forwards"]) == 2 and d["iters"] > 0
    # the step profile says what an iteration cost and carried
    prof = d["step_profile_rank0"]
    assert prof and all(v["n"] > 0 and v["p50_ms"] >= 0 for v in prof.values())

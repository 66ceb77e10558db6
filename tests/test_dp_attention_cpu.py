"""Data-parallel attention + expert-parallel MoE (DeepSeek-V3-shaped MLA
model) on 2 gloo ranks: every rank serves its own prompts with E/2 experts,
ranks stay in lockstep (idle forwards), and the greedy outputs equal a
single engine holding every expert."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_dp_attention_ep_two_ranks_cpu():
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29793", "-m",
           "infera_b200.bench.dp_check", "--cpu", "--prompts", "3"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    res = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    assert res["agreement"] >= 0.95, res
    # 3 prompts over 2 ranks: rank 1 runs out of work first and idles in step
    assert any(rk["idle_forwards"] > 0 for rk in res["ranks"]), res

"""Prefill/decode pair of tensor-parallel instances on 2 gloo ranks: the
leader adopts page plans, push completions and resumes as commands that
every rank applies at the same step; each prefill rank pushes its KV-head
shard into the same rank of the decode group (one request layer by layer,
one after its prompt); the decode outputs equal a mixed tensor-parallel
instance's and the decode group computes only each prompt's last token."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pd_pair_of_tp2_instances_cpu():
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29795", "-m",
           "infera_b200.bench.pd_tp_check", "--cpu"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    res = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    assert res["equal_to_mixed"], res
    for rk in res["ranks"]:
        assert rk["pushes"] == 2 and rk["layerwise"] == 1 and rk["decode_prompt_tokens"] == 2, res
        assert not rk["unfinished"], res

"""Expert parallelism over 2 gloo ranks on CPU: the EP MoE layer (routing,
count / row all-to-alls, regroup, grouped experts, return, combine) equals
the single-device layer on the same tokens."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_ep_two_ranks_cpu():
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29763", "-m",
           "infera_b200.bench.ep_check", "--cpu", "--tokens", "23", "--hidden", "64", "--ffn", "32", "--experts", "8",
           "--top-k", "2"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=300)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    assert '"max_rel_err"' in out

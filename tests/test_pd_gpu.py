"""Prefill/decode KV push on the GPU: two engines in one process, on one GPU
(local stores) and on two GPUs (peer stores over NVLink); the decode output
must equal a single engine's, and the pushed pages must be exactly the
prefill's."""

import pytest
import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _eng(dev, **kw):
    return LLMEngine(EngineConfig(model="tiny-dense-gpu", use_cuda_graphs=False, num_pages=512, **kw), device=dev)


def _pair(pre, dec, prompt, n, room):
    ep = dec.pd_rendezvous.endpoint
    dec.add_request(f"d{room}", prompt, SamplingParams(max_tokens=n, ignore_eos=True,
                                                       kv_transfer={"do_remote_prefill": True, "room": room}))
    pre.add_request(f"p{room}", prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                                       kv_transfer={"do_remote_decode": True, "room": room,
                                                                    "decode_kv_endpoint": ep}))
    out = []
    for _ in range(2000):
        if pre.has_unfinished():
            torch.cuda.set_device(pre.device)
            pre.step()
        if dec.has_unfinished():
            torch.cuda.set_device(dec.device)
            for o in dec.step():
                out.extend(o.new_token_ids)
        if not dec.has_unfinished() and not pre.has_unfinished():
            break
    return out


@pytest.mark.parametrize("devs", [("cuda:0", "cuda:0"), ("cuda:0", "cuda:1")])
def test_pd_push(devs):
    if torch.cuda.device_count() < len(set(devs)):
        pytest.skip("needs 2 GPUs")
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, 4000, (300,), generator=g).tolist()
    ref = _eng("cuda:0").generate([prompt], SamplingParams(max_tokens=8, ignore_eos=True))[0]
    pre = _eng(devs[0], disagg_mode="prefill")
    dec = _eng(devs[1], disagg_mode="decode", kv_push_endpoint=f"local://pd-gpu-{devs[1]}")
    out = _pair(pre, dec, prompt, 8, 5)
    assert pre.pd_agent.stats["pushes"] == 1
    assert dec.pd_rendezvous.stats["done"] == 1 and dec.counters["prompt_tokens"] == 1
    torch.cuda.set_device(dec.device)
    assert K.scratch(dec.device).read_status() == 0
    agree = sum(a == b for a, b in zip(out, ref)) / len(ref)
    assert len(out) == 8 and agree >= 0.75, (out, ref)


@pytest.mark.parametrize("channels", [1, 2])
def test_page_copy_and_push_kernels(channels):
    """ib_kv_page_copy (gather / scatter) and ib_kv_push_pages on a K/V pair
    and on a latent (one-channel, 576-wide) cache: bit-exact page moves."""
    L, slots, H = 3, 64 * 16, 576 if channels == 1 else 256
    g = torch.Generator().manual_seed(2)
    k = torch.randn(L, slots, H, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(L, slots, H, generator=g).to(torch.bfloat16).cuda() if channels == 2 else \
        torch.zeros(L, 1, 1, dtype=torch.bfloat16, device="cuda")
    pages = torch.tensor([5, 0, 63, 17], dtype=torch.int32, device="cuda")
    chunk = torch.empty(channels * L * 4 * 16 * H, dtype=torch.bfloat16, device="cuda")
    K.kv_page_copy(k, v, chunk, pages, gather=True)
    idx = (pages.long()[:, None] * 16 + torch.arange(16, device="cuda")).reshape(-1)
    view = chunk.view(channels, L, 64, H)
    assert torch.equal(view[0], k[:, idx])
    if channels == 2:
        assert torch.equal(view[1], v[:, idx])
    k2, v2 = torch.zeros_like(k), torch.zeros_like(v)
    K.kv_page_copy(k2, v2, chunk, pages, gather=False)
    assert torch.equal(k2[:, idx], k[:, idx])
    dk, dv = torch.zeros_like(k), torch.zeros_like(v)
    dst = torch.tensor([1, 2, 3, 60], dtype=torch.int32, device="cuda")
    K.kv_push_pages(k, v, dk, dv, pages, dst, layers=(1, 3))
    torch.cuda.synchronize()
    idx_d = (dst.long()[:, None] * 16 + torch.arange(16, device="cuda")).reshape(-1)
    assert torch.equal(dk[1:3, idx_d], k[1:3, idx]) and int(dk[0].abs().sum()) == 0
    if channels == 2:
        assert torch.equal(dv[1:3, idx_d], v[1:3, idx])
    else:
        assert int(dv.abs().sum()) == 0


def test_pd_pair_of_tp2_instances():
    """The tensor-parallel PD protocol on 2 GPUs (fused TP all-reduce, NCCL
    fence after the pushes): decode outputs equal a mixed TP instance's."""
    import json
    import os
    import subprocess
    import sys

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29796", "-m",
           "infera_b200.bench.pd_tp_check", "--model", "tiny-dense-gpu"]
    r = subprocess.run(cmd, env=dict(os.environ, PYTHONPATH=root, NCCL_NVLS_ENABLE="0"), cwd=root,
                       stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=360)
    out = r.stdout.decode()
    assert r.returncode == 0, out[-3000:]
    res = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    agree = sum(x == y for o, f in zip(res["outputs"], res["reference"]) for x, y in zip(o, f))
    assert agree >= 0.8 * sum(len(f) for f in res["reference"]), res
    for rk in res["ranks"]:
        assert rk["pushes"] == 2 and rk["decode_prompt_tokens"] == 2 and not rk["unfinished"], res

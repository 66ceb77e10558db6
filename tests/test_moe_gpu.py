"""MoE kernels against the fp32 PyTorch oracle (the CPU paths): grouped
top-k routing, expert permutation, the tcgen05 grouped GEMM (plain and
SwiGLU, several token-tile widths, empty experts) and the whole layer."""

import pytest
import torch

from infera_b200.models.moe import MoELayer
from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-6))


def _status():
    assert K.scratch(torch.device("cuda", 0)).read_status() == 0


def test_topk_matches_oracle():
    torch.manual_seed(0)
    T, E = 300, 256
    logits = torch.randn(T, E)
    bias = torch.randn(E) * 0.05
    ids_c, w_c = K.moe_topk(logits, 8, n_groups=8, topk_groups=4, bias=bias, scaling=2.5)
    ids_g, w_g = K.moe_topk(logits.cuda(), 8, n_groups=8, topk_groups=4, bias=bias.cuda(), scaling=2.5)
    torch.cuda.synchronize()
    for t in range(T):
        assert sorted(ids_g[t].tolist()) == sorted(ids_c[t].tolist())
    # weights per expert
    wg = torch.zeros(T, E).scatter_(1, ids_g.cpu().long(), w_g.cpu())
    wc = torch.zeros(T, E).scatter_(1, ids_c.long(), w_c)
    assert _rel(wg, wc) < 1e-4


def test_permute_consistent():
    torch.manual_seed(1)
    T, k, E = 257, 8, 64
    ids = torch.randint(0, E, (T, k), dtype=torch.int32)
    off_c, _, _ = K.moe_permute(ids, E)
    off, ros, tor = K.moe_permute(ids.cuda(), E)
    torch.cuda.synchronize()
    assert torch.equal(off.cpu(), off_c)
    ros, tor, off = ros.cpu().long(), tor.cpu().long(), off.cpu().long()
    assert sorted(ros.tolist()) == list(range(T * k))
    for i in range(T * k):
        e = int(ids.view(-1)[i])
        assert off[e] <= ros[i] < off[e + 1] and tor[ros[i]] == i // k


@pytest.mark.parametrize("counts,swiglu,bn", [
    ([5, 0, 17, 1, 40, 0, 3, 130], False, None), ([5, 0, 17, 1, 40, 0, 3, 130], True, None),
    ([200, 1, 0, 64, 63, 65, 0, 9], True, 64), ([1] * 8, False, 16), ([300, 0, 0, 0, 0, 0, 0, 257], True, 128),
])
def test_grouped_gemm(counts, swiglu, bn):
    torch.manual_seed(2)
    E, N, Kd = len(counts), 256, 512
    R = sum(counts)
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.cumsum(torch.tensor(counts), 0).to(torch.int32)
    x = (torch.randn(R, Kd) * 0.5).to(torch.bfloat16)
    w = (torch.randn(E, N, Kd) / Kd ** 0.5).to(torch.bfloat16)
    ref = K.gemm_grouped(x, w, off, swiglu=swiglu)
    out = K.gemm_grouped(x.cuda(), w.cuda(), off.cuda(), swiglu=swiglu, bn=bn)
    torch.cuda.synchronize()
    _status()
    assert out.shape == ref.shape and _rel(out.cpu(), ref) < 1e-2


@pytest.mark.parametrize("T", [1, 33, 257])
def test_moe_layer(T):
    torch.manual_seed(3)
    layer = MoELayer(hidden=1024, moe_ffn=512, num_experts=32, top_k=4, n_groups=4, topk_groups=2,
                     routed_scaling=2.5, num_shared=1, device="cpu", seed=3)
    x = torch.randn(T, 1024).to(torch.bfloat16)
    ids, wts = layer.route(x)
    ref = layer.forward(x, ids, wts)
    g = layer.to("cuda")
    out = g.forward(x.cuda(), ids.cuda(), wts.cuda())
    torch.cuda.synchronize()
    _status()
    assert _rel(out.cpu(), ref) < 2e-2


def test_engine_moe_model_with_graphs():
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams
    from infera_b200.models.reference import reference_logits

    eng = LLMEngine(EngineConfig(model="tiny-moe-gqa-gpu", num_pages=256, max_num_seqs=16), device="cuda:0")
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 4000, (n,), generator=g).tolist() for n in (7, 65, 200)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    _status()
    assert [len(o) for o in outs] == [6, 6, 6]
    # the first sampled token is the argmax of the oracle's last-position logits
    # unless the top two are within rounding
    for p, o in zip(prompts, outs):
        lg = reference_logits(eng.model, p)[-1]
        top = torch.topk(lg, 2)
        assert o[0] == int(top.indices[0]) or float(top.values[0] - top.values[1]) < 0.05

"""W8A8 e4m3 GEMM with UE8M0 block scales (tcgen05 kind::mxf8f6f4
block_scale) and the activation quantiser, against plain PyTorch fp32
computations of the same ops."""

import pytest
import torch

from infera_b200.ops import fp8
from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


def test_act_quant_matches_cpu_bitwise():
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(37, 1024, device="cuda", generator=g) * 5).to(torch.bfloat16)
    x[3] = 0
    x[5, :128] *= 1000
    q, sf = fp8.quant_act(x)
    qc, sfc = fp8.quant_act(x.cpu())
    assert torch.equal(sf[:, :37].cpu(), sfc)
    assert torch.equal(q.cpu().view(torch.uint8), qc.view(torch.uint8))
    assert K.scratch().read_status() == 0


@pytest.mark.parametrize("M,N,Kd", [(1, 256, 1024), (7, 2560, 8192), (32, 1024, 512), (100, 768, 2048),
                                    (192, 512, 1024), (300, 1280, 4096), (1024, 2048, 1024)])
def test_gemm_fp8_matches_fp32(M, N, Kd):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    w = fp8.quantize_weight(torch.randn(N, Kd, device="cuda", generator=g) * 0.03)
    x = torch.randn(M, Kd, device="cuda", generator=g).to(torch.bfloat16)
    q, sf = fp8.quant_act(x)
    y = fp8.gemm_fp8(q, sf, w)
    torch.cuda.synchronize()
    ref = fp8.dequant_act(q.cpu(), sf.cpu()) @ w.to("cpu").dequant().t()
    assert _rel(y.cpu(), ref) < 1e-2
    assert K.scratch().read_status() == 0


def test_gemm_fp8_swiglu_and_linear():
    g = torch.Generator(device="cuda").manual_seed(5)
    w = fp8.quantize_weight(torch.randn(1024, 2048, device="cuda", generator=g) * 0.03)
    x = torch.randn(48, 2048, device="cuda", generator=g).to(torch.bfloat16)
    y = K.linear(x, w, swiglu=True)  # dispatches on the fp8 weight
    q, sf = fp8.quant_act(x.cpu())
    r = fp8.dequant_act(q, sf) @ w.to("cpu").dequant().t()
    ref = torch.nn.functional.silu(r[:, 0::2]) * r[:, 1::2]
    assert y.shape == (48, 512)
    assert _rel(y.cpu(), ref) < 1e-2
    assert K.scratch().read_status() == 0


def test_gemm_fp8_grouped_matches_loop():
    g = torch.Generator(device="cuda").manual_seed(9)
    E, N, Kd = 6, 256, 1024
    w = fp8.quantize_weight(torch.randn(E * N, Kd, device="cuda", generator=g) * 0.03)
    counts = torch.tensor([0, 5, 40, 1, 0, 77])
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.cumsum(counts, 0)
    R = int(off[-1])
    x = torch.randn(R, Kd, device="cuda", generator=g).to(torch.bfloat16)
    for swiglu in (False, True):
        y = fp8.gemm_fp8_grouped(x, w, E, off.cuda(), swiglu=swiglu)
        ref = fp8.gemm_fp8_grouped(x.cpu(), w.to("cpu"), E, off, swiglu=swiglu)
        assert _rel(y.cpu(), ref) < 1e-2
    assert K.scratch().read_status() == 0


@pytest.mark.parametrize("graphs", [False, True])
def test_fp8_engine_matches_oracle(graphs):
    """The dense decoder with e4m3 block-scaled weights (every projection
    through ib_gemm_fp8) against the CPU oracle that quantises alike."""
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams
    from infera_b200.models.reference import reference_greedy

    cfg = EngineConfig(model="tiny-dense-fp8-gpu", num_pages=128, max_num_seqs=8, max_batched_tokens=96,
                       use_cuda_graphs=graphs)
    eng = LLMEngine(cfg, device="cuda:0")
    assert not isinstance(eng.model.w.layers[0]["qkv"], torch.Tensor)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (5, 130, 47)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    for p, o in zip(prompts, outs):
        ref, margins = reference_greedy(eng.model, p, 6)
        for i, (a, b) in enumerate(zip(o, ref)):
            if a != b:
                assert margins[i] < 0.3, (i, a, b, margins[i])
                break

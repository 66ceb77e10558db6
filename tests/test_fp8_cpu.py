"""fp8 block-scaled format on CPU: power-of-two scales, e4m3 range,
quantisation error bounds, and the PyTorch paths of the W8A8 GEMMs against
a plain fp32 matmul of the dequantised operands."""

import torch

from infera_b200.ops import fp8


def test_weight_quant_format():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 512, generator=g) * 0.02
    w[:128, :128] *= 50  # one block with a much larger range
    qw = fp8.quantize_weight(w)
    assert qw.q.dtype == torch.float8_e4m3fn and qw.q.shape == (300, 512)
    assert qw.sf.shape == (3, 4) and qw.sf.dtype == torch.uint8
    assert qw.q.float().abs().max() <= 448
    # each scale is the smallest power of two that fits the block
    d = qw.dequant()
    rel = (d - w).norm() / w.norm()
    assert rel < 0.04, rel
    assert qw.sf[0, 0] > qw.sf[0, 1]


def test_exponent_rule():
    amax = torch.tensor([0.0, 448.0, 449.0, 224.0, 1.0, 896.0])
    e = fp8._exp_pow2(amax)
    assert e.tolist() == [0, 0, 1, -1, -8, 1]


def test_act_quant_layout_and_roundtrip():
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(5, 384, generator=g) * 3).to(torch.bfloat16)
    q, sf = fp8.quant_act(x)
    assert q.shape == (5, 384) and sf.shape == (3, 5)
    d = fp8.dequant_act(q, sf)
    assert ((d - x.float()).norm() / x.float().norm()) < 0.04


def test_gemm_fp8_cpu_matches_dequantised_fp32():
    g = torch.Generator().manual_seed(2)
    w = fp8.random_weight(256, 256, 0.05, generator=g)
    x = torch.randn(7, 256, generator=g).to(torch.bfloat16)
    q, sf = fp8.quant_act(x)
    y = fp8.gemm_fp8(q, sf, w)
    ref = fp8.dequant_act(q, sf) @ w.dequant().t()
    assert ((y.float() - ref).norm() / ref.norm()) < 1e-2
    ys = fp8.gemm_fp8(q, sf, w, swiglu=True)
    refs = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
    assert ys.shape == (7, 128)
    assert ((ys.float() - refs).norm() / refs.norm()) < 1e-2


def test_weight_slicing():
    g = torch.Generator().manual_seed(3)
    w = fp8.random_weight(512, 384, 0.05, generator=g)
    r = w.rows(128, 384)
    assert torch.equal(r.dequant(), w.dequant()[128:384])
    c = w.cols(128, 384)
    assert torch.equal(c.dequant(), w.dequant()[:, 128:384])


def test_fp8_engine_cpu_matches_oracle():
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams
    from infera_b200.models.reference import reference_greedy

    eng = LLMEngine(EngineConfig(model="tiny-dense-fp8", use_cuda_graphs=False, num_pages=64,
                                 max_batched_tokens=24, max_num_seqs=4), device="cpu")
    assert isinstance(eng.model.w.layers[0]["down"], fp8.FP8Weight)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 40)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))
    for p, o in zip(prompts, outs):
        ref, margins = reference_greedy(eng.model, p, 5)
        for i, (a, b) in enumerate(zip(o, ref)):
            if a != b:
                assert margins[i] < 0.1, (i, a, b, margins[i])
                break

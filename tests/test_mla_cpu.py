"""DeepSeek-V3-shaped MLA + MoE decoder on CPU: the engine (absorbed MLA
over the paged latent cache, chunked prefill, decode) against a plain fp32
forward that expands the latent into per-head keys and values."""

import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.models.mla import MLAModel, reference_logits_mla
from infera_b200.ops import mla as M


def _greedy_ref(model, prompt, n):
    toks = list(prompt)
    out, margins = [], []
    for _ in range(n):
        lg = reference_logits_mla(model, toks)[-1]
        top = torch.topk(lg, 2)
        out.append(int(top.indices[0]))
        margins.append(float(top.values[0] - top.values[1]))
        toks.append(out[-1])
    return out, margins


def test_mla_attention_cpu_matches_expanded():
    g = torch.Generator().manual_seed(0)
    hq, L = 4, 40
    cache = torch.randn(64, 96, generator=g).to(torch.bfloat16)
    bt = torch.tensor([[3, 1, 2, 0]], dtype=torch.int32)
    q = torch.randn(1, hq, 96, generator=g).to(torch.bfloat16)
    o = M.mla_attention(q, cache, bt, torch.tensor([0]), torch.tensor([L]), 0.1, rope_dim=32)
    slots = torch.cat([torch.arange(16) + 16 * p for p in (3, 1, 2)])[:L]
    kv = cache[slots].float()
    ref = torch.softmax(q[0].float() @ kv.t() * 0.1, -1) @ kv[:, :64]
    assert torch.allclose(o[0].float(), ref, atol=2e-2, rtol=2e-2)


def test_mla_engine_matches_reference():
    eng = LLMEngine(EngineConfig(model="tiny-moe", use_cuda_graphs=False, num_pages=64, max_batched_tokens=24,
                                 max_num_seqs=4), device="cpu")
    assert isinstance(eng.model, MLAModel)
    assert eng.runner.v_cache.numel() == eng.model.cfg.num_layers
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 37)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))
    assert [len(o) for o in outs] == [5, 5]
    for p, o in zip(prompts, outs):
        ref, margins = _greedy_ref(eng.model, p, 5)
        for i, (a, b) in enumerate(zip(o, ref)):
            if a != b:
                assert margins[i] < 0.05, (i, a, b, margins[i])
                break

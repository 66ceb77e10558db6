"""MoE routing and expert computation, CPU paths (the fp32 oracle of the
GPU kernels): grouped top-k semantics, permutation, grouped GEMM, combine."""

import torch

from infera_b200.models.moe import MoELayer
from infera_b200.ops import kernels as K


def test_grouped_topk_semantics():
    torch.manual_seed(0)
    T, E = 5, 16
    logits = torch.randn(T, E)
    ids, w = K.moe_topk(logits, top_k=3, n_groups=4, topk_groups=2, scaling=2.0)
    s = torch.sigmoid(logits)
    for t in range(T):
        groups = s[t].view(4, 4).topk(2, -1).values.sum(-1).topk(2).indices.tolist()
        allowed = [g * 4 + i for g in groups for i in range(4)]
        assert all(int(e) in allowed for e in ids[t])
        assert abs(float(w[t].sum()) - 2.0) < 1e-5
    ids1, _ = K.moe_topk(logits, top_k=3)
    assert torch.equal(ids1.long(), torch.sigmoid(logits).topk(3, -1).indices)


def test_permute_and_layer_match_dense_computation():
    torch.manual_seed(1)
    layer = MoELayer(hidden=64, moe_ffn=32, num_experts=8, top_k=2, device="cpu", num_shared=1)
    x = torch.randn(11, 64).to(torch.bfloat16)
    ids, wts = layer.route(x)
    offsets, row_of_slot, token_of_row = K.moe_permute(ids, 8)
    assert int(offsets[-1]) == 22 and sorted(row_of_slot.tolist()) == list(range(22))
    assert all(int(token_of_row[int(row_of_slot[i])]) == i // 2 for i in range(22))
    y = layer.forward(x, ids, wts)
    ref = torch.zeros(11, 64)
    for t in range(11):
        for j in range(2):
            e = int(ids[t, j])
            h = x[t].float() @ layer.w13[e].float().t()
            a = torch.nn.functional.silu(h[0::2]) * h[1::2]
            ref[t] += float(wts[t, j]) * (a.to(torch.bfloat16).float() @ layer.w2[e].float().t())
    hs = x.float() @ layer.shared[0].float().t()
    ref += (torch.nn.functional.silu(hs[:, 0::2]) * hs[:, 1::2]).to(torch.bfloat16).float() @ layer.shared[1].float().t()
    assert float((y.float() - ref).norm() / ref.norm()) < 2e-2


def test_engine_serves_moe_model():
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams
    from infera_b200.models.reference import reference_greedy

    eng = LLMEngine(EngineConfig(model="tiny-moe-gqa", use_cuda_graphs=False, num_pages=64, max_batched_tokens=24),
                    device="cpu")
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (9, 30)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=5, ignore_eos=True))
    for p, o in zip(prompts, outs):
        ref, margins = reference_greedy(eng.model, p, 5)
        for i, (a, b) in enumerate(zip(o, ref)):
            if a != b:
                assert margins[i] < 0.05, (i, a, b, margins[i])
                break

"""MLA kernels on a B200 against PyTorch fp32 computations of the same ops:
the absorbed latent attention (tcgen05, value halves, key splits + merge),
the fused latent-row write (RMSNorm + RoPE + cache store), and the
DeepSeek-V3-shaped engine (fp8 projections, grouped absorptions, routed
experts) against the expanded fp32 oracle."""

import pytest
import torch

from infera_b200.ops import kernels as K
from infera_b200.ops import mla as M

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


@pytest.mark.parametrize("hq,lens,splits,contig", [(128, [1, 33, 500], 1, False), (16, [7, 64, 2049], 1, False),
                                                   (128, [3000, 17], 4, False), (64, [0, 100, 4096], 8, False),
                                                   (128, [1000, 4096, 129], 2, True),
                                                   (128, [2048, 300], None, True)])
def test_mla_attention_matches_fp32(hq, lens, splits, contig):
    """contig: each sequence's pages consecutive (eight-page runs load as one box)."""
    g = torch.Generator(device="cuda").manual_seed(hq + len(lens))
    B = len(lens)
    pages_per = max(1, max(-(-L // 16) for L in lens))
    n_pages = B * pages_per + 3
    cache = torch.randn(n_pages * 16, 576, device="cuda", generator=g).to(torch.bfloat16)
    if contig:
        perm = torch.arange(1, n_pages, device="cuda", dtype=torch.int32)
    else:
        perm = torch.randperm(n_pages, device="cuda", generator=g).to(torch.int32)
    bt = perm[: B * pages_per].view(B, pages_per).contiguous()
    q = (torch.randn(B, hq, 576, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    rows = torch.arange(B, dtype=torch.int32, device="cuda")
    kvl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    o = M.mla_attention(q, cache, bt, rows, kvl, 0.07, splits=splits)
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    ref = M.mla_attention(q.cpu(), cache.cpu(), bt.cpu(), rows.cpu(), kvl.cpu(), 0.07)
    for i, L in enumerate(lens):
        if L == 0:
            assert float(o[i].float().abs().max()) == 0.0
        else:
            assert _rel(o[i].cpu(), ref[i]) < 2e-2, (i, L)


def test_mla_rope_kvwrite_matches_fp32():
    g = torch.Generator(device="cuda").manual_seed(1)
    T, hq = 9, 32
    q = torch.randn(T, hq, 576, device="cuda", generator=g).to(torch.bfloat16)
    kva = torch.randn(T, 576, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(512, device="cuda", generator=g)).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 2, 100, 5, 6, 7, 4000, 9], dtype=torch.int32, device="cuda")
    slots = torch.tensor([3, 4, 5, -1, 7, 8, 9, 10, 0], dtype=torch.int32, device="cuda")
    cs = K.rope_cos_sin(4096, 64, 10000.0, None, device="cuda")
    cache = torch.zeros(16, 576, dtype=torch.bfloat16, device="cuda")
    qc, cc = q.cpu().clone(), cache.cpu().clone()
    M.mla_rope_kvwrite(q, kva, pos, slots, cs, w, 1e-6, cache)
    M.mla_rope_kvwrite(qc, kva.cpu(), pos.cpu(), slots.cpu(), cs.cpu(), w.cpu(), 1e-6, cc)
    torch.cuda.synchronize()
    assert (q.cpu().float() - qc.float()).abs().max() < 3e-2
    assert (cache.cpu().float() - cc.float()).abs().max() < 3e-2
    assert float(cache[6].float().abs().max()) == 0.0  # slot -1 wrote nothing


def test_mla_engine_matches_oracle():
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams
    from infera_b200.models.mla import reference_logits_mla

    eng = LLMEngine(EngineConfig(model="tiny-mla-gpu", num_pages=128, max_num_seqs=4, max_batched_tokens=256,
                                 use_cuda_graphs=False), device="cuda:0")
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (6, 90)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=4, ignore_eos=True))
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    assert [len(o) for o in outs] == [4, 4]
    # last-step logits of a fresh single prompt against the expanded oracle
    p = prompts[1] + outs[1]
    eng.generate([p], SamplingParams(max_tokens=1, ignore_eos=True))
    lg = eng.runner.last_logits[0].float().cpu()
    ref = reference_logits_mla(eng.model, p)[-1]
    cc = torch.corrcoef(torch.stack([lg, ref]))[0, 1]
    assert cc > 0.995, float(cc)


@pytest.mark.parametrize("hq,q_lens,ctx_lens", [(128, [300, 128], [300, 1000]), (16, [1, 257, 64], [4097, 257, 64]),
                                                (32, [513], [2000])])
def test_mla_prefill_unabsorbed_matches_fp32(hq, q_lens, ctx_lens):
    """Prompt chunks through the gathered latent -> [k_nope | v] GEMM -> flash
    attention over 128 + 64 score dims, against the CPU restatement of the
    same math (fp32), with permuted pages, table rows and prior context."""
    g = torch.Generator(device="cuda").manual_seed(hq + sum(q_lens))
    B = len(q_lens)
    pages_per = max(-(-c // 16) for c in ctx_lens)
    n_pages = B * pages_per + 5
    cache = (torch.randn(n_pages * 16, 576, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    perm = torch.randperm(n_pages, device="cuda", generator=g).to(torch.int32)
    bt = torch.zeros(B + 2, pages_per, dtype=torch.int32, device="cuda")
    rows = torch.arange(B, dtype=torch.int32, device="cuda").flip(0) + 1          # table rows 1..B, reversed
    bt[rows.long()] = perm[: B * pages_per].view(B, pages_per)
    Tp = sum(q_lens)
    qb = (torch.randn(Tp, hq * 192, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    q_full = (torch.randn(Tp, hq, 576, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w_uk = (torch.randn(hq, 512, 128, device="cuda", generator=g) / 512 ** 0.5).to(torch.bfloat16)
    w_uv = (torch.randn(hq, 128, 512, device="cuda", generator=g) / 512 ** 0.5).to(torch.bfloat16)
    w_up = M.kv_up_weight(w_uk, w_uv)
    starts = [0]
    for n in q_lens[:-1]:
        starts.append(starts[-1] + n)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    tiles = i32(K.prefill_tiles(q_lens, 128)).view(-1, 2)
    args = (cache, bt, rows, (q_lens, ctx_lens), i32(starts), i32(q_lens), i32(ctx_lens), tiles)
    out = M.mla_prefill(qb, q_full, *args, w_up, hq, 128, 128, 0.07)
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    cpu = lambda t: t.cpu() if isinstance(t, torch.Tensor) else t  # noqa: E731
    ref = M.mla_prefill(qb.cpu(), q_full.cpu(), *[cpu(a) for a in args], w_up.cpu(), hq, 128, 128, 0.07)
    assert _rel(out.cpu(), ref) < 2e-2

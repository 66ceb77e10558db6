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


def _mla(**kw):
    return LLMEngine(EngineConfig(model="tiny-moe", use_cuda_graphs=False, max_num_seqs=4, **kw), device="cpu")


def test_mla_latent_cache_tier_save_and_promote():
    """A latent cache (one channel) saves to and promotes from the host tier;
    the chunk header records one KV channel."""
    eng = _mla(num_pages=12, max_batched_tokens=256, kv_tier="host:0.05")
    assert eng.tier.C == 1
    g = torch.Generator().manual_seed(4)
    a = torch.randint(0, 1000, (64,), generator=g).tolist()
    sp = SamplingParams(max_tokens=2, ignore_eos=True)
    eng.generate([a], sp)
    for _ in range(3):
        eng.generate([torch.randint(0, 1000, (64,), generator=g).tolist()], sp)
    eng.tier.flush()
    assert eng.tier.stats["saved"] >= 4
    a2 = a + [5, 6, 7]
    out = eng.generate([a2], SamplingParams(max_tokens=3, ignore_eos=True))[0]
    assert eng.bm.stats["tier_hit_tokens"] >= 48
    ref, margins = _greedy_ref(eng.model, a2, 3)
    for i, (x, y) in enumerate(zip(out, ref)):
        if x != y:
            assert margins[i] < 0.05
            break


def test_mla_latent_cache_pd_push():
    """Prefill -> decode push of a latent cache, whole and layer by layer:
    the decode output equals a single engine's."""
    import time

    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, 1024, (70,), generator=g).tolist()
    ref = _mla(num_pages=64, max_batched_tokens=128).generate([prompt], SamplingParams(max_tokens=4,
                                                                                       ignore_eos=True))[0]
    for room, chunk in ((41, 128), (42, 24)):   # one forward (whole push) / several chunks (layer-wise)
        dec = _mla(num_pages=64, max_batched_tokens=128, disagg_mode="decode",
                   kv_push_endpoint=f"local://pd-mla-{room}")
        pre = _mla(num_pages=64, max_batched_tokens=chunk, disagg_mode="prefill")
        dec.add_request("d", prompt, SamplingParams(max_tokens=4, ignore_eos=True,
                                                    kv_transfer={"do_remote_prefill": True, "room": room}))
        dec.step()
        pre.add_request("p", prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                                    kv_transfer={"do_remote_decode": True, "room": room,
                                                                 "decode_kv_endpoint": dec.pd_rendezvous.endpoint}))
        out = []
        for _ in range(500):
            if pre.has_unfinished():
                pre.step()
                time.sleep(0.01)
            if dec.has_unfinished():
                for o in dec.step():
                    out.extend(o.new_token_ids)
            if not dec.has_unfinished() and not pre.has_unfinished():
                break
        assert out == ref, room
        assert pre.pd_agent.stats["pushes"] == 1 and dec.counters["prompt_tokens"] == 1
        L, _, H = pre.runner.k_cache.shape
        assert pre.pd_agent.stats["bytes"] == pre.pd_agent.stats["pages"] * 16 * L * H * 2   # one channel


def test_pd_refuses_a_mismatched_decode_cache():
    import pytest

    dec = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=32, disagg_mode="decode",
                                 kv_push_endpoint="local://pd-mla-mismatch"), device="cpu")
    pre = _mla(num_pages=32, max_batched_tokens=128, disagg_mode="prefill")
    from infera_b200.engine.pd import PDPushAgent

    agent = PDPushAgent(pre)
    with pytest.raises(RuntimeError, match="channels"):
        agent._peer(dec.pd_rendezvous.endpoint)


def test_mla_prefill_unabsorbed_cpu_matches_absorbed_attention():
    """The non-absorbed prompt path (gathered latent -> per-head [k_nope | v]
    -> 128 + rope score dims) equals the absorbed latent attention followed
    by the W_UV projection, with prior context and permuted pages."""
    g = torch.Generator().manual_seed(5)
    hq, L, dn, dv, dr = 4, 64, 32, 32, 32
    q_lens, ctx_lens = [5, 19], [40, 19]
    bt = torch.tensor([[0, 0, 0], [4, 2, 7], [1, 5, 3]], dtype=torch.int32)
    rows = torch.tensor([2, 1], dtype=torch.int32)
    cache = torch.randn(8 * 16, L + dr, generator=g).to(torch.bfloat16)
    w_uk = (torch.randn(hq, L, dn, generator=g) / L ** 0.5).to(torch.bfloat16)
    w_uv = (torch.randn(hq, dv, L, generator=g) / L ** 0.5).to(torch.bfloat16)
    Tp = sum(q_lens)
    qb = torch.randn(Tp, hq * (dn + dr), generator=g).to(torch.bfloat16)
    q_rope = torch.randn(Tp, hq, L + dr, generator=g).to(torch.bfloat16)
    t = lambda v: torch.tensor(v, dtype=torch.int32)  # noqa: E731
    out = M.mla_prefill(qb, q_rope, cache, bt, rows, (q_lens, ctx_lens), t([0, 5]), t(q_lens), t(ctx_lens),
                        t([[0, 0], [1, 0]]), M.kv_up_weight(w_uk, w_uv), hq, dn, dv, 0.1, dr=dr)
    # absorbed: q_lat = W_UK q_nope, attention over the latent rows, then W_UV
    qn = qb.float().view(Tp, hq, dn + dr)[:, :, :dn]
    q_abs = torch.cat([torch.einsum("thd,hld->thl", qn, w_uk.float()), q_rope.float()[:, :, L:]], -1)
    row_of = torch.cat([rows[i].repeat(n) for i, n in enumerate(q_lens)])
    kvlen = torch.cat([torch.arange(c - n, c) + 1 for n, c in zip(q_lens, ctx_lens)])
    o_lat = M.mla_attention(q_abs.to(torch.bfloat16), cache, bt, row_of, kvlen, 0.1, rope_dim=dr)
    ref = torch.einsum("thl,hvl->thv", o_lat.float(), w_uv.float()).reshape(Tp, hq * dv)
    err = float((out.float() - ref).norm() / ref.norm())
    assert err < 3e-2, err

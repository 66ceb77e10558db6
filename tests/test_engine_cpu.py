"""Engine correctness on CPU (the torch restatement of every kernel):
chunked prefill, prefix-cache reuse, decode and preemption must give the
same greedy tokens as a plain full-sequence forward."""

import torch

from infera_b200.engine.block_manager import BlockManager
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.models.reference import reference_greedy
from infera_b200.utils.hashing import chain_hashes, hash_chunk


def _engine(**kw):
    cfg = EngineConfig(model="tiny-dense", use_cuda_graphs=False, **kw)
    return LLMEngine(cfg, device="cpu")


def _check_against_reference(eng, prompts, outs, n):
    for p, o in zip(prompts, outs):
        ref, margins = reference_greedy(eng.model, p, n)
        for i, (a, b) in enumerate(zip(o, ref)):
            if a != b:
                # a flip is only acceptable on a near-tie of the reference
                assert margins[i] < 0.05, (i, a, b, margins[i])
                break


def test_generate_matches_reference_with_chunking():
    eng = _engine(num_pages=64, max_batched_tokens=24, max_num_seqs=4)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 40, 17)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    assert [len(o) for o in outs] == [6, 6, 6]
    _check_against_reference(eng, prompts, outs, 6)


def test_prefix_cache_hit_and_reuse():
    eng = _engine(num_pages=64, max_batched_tokens=256, max_num_seqs=4)
    g = torch.Generator().manual_seed(2)
    prefix = torch.randint(0, 1024, (48,), generator=g).tolist()
    p1 = prefix + [1, 2, 3]
    p2 = prefix + [7, 8, 9, 10]
    o1 = eng.generate([p1], SamplingParams(max_tokens=3, ignore_eos=True))[0]
    assert eng.bm.stats["hit_tokens"] == 0
    o2 = eng.generate([p2], SamplingParams(max_tokens=3, ignore_eos=True))[0]
    assert eng.bm.stats["hit_tokens"] == 48
    _check_against_reference(eng, [p1, p2], [o1, o2], 3)
    # a later turn that extends p1 + its output reuses everything computed
    p3 = p1 + o1 + [11, 12]
    before = eng.bm.stats["hit_tokens"]
    o3 = eng.generate([p3], SamplingParams(max_tokens=2, ignore_eos=True))[0]
    assert eng.bm.stats["hit_tokens"] - before == (len(p1) + len(o1)) // 16 * 16
    _check_against_reference(eng, [p3], [o3], 2)


def test_preemption_recomputes_correctly():
    # 6 pages of 16 tokens cannot hold three 40-token sequences at once
    eng = _engine(num_pages=9, max_batched_tokens=64, max_num_seqs=4, enable_prefix_cache=False)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1024, (30,), generator=g).tolist() for _ in range(3)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))
    assert all(len(o) == 12 for o in outs)
    _check_against_reference(eng, prompts, outs, 12)


def test_block_manager_events_and_eviction():
    events = []
    bm = BlockManager(num_pages=5, page_size=4, event_sink=lambda k, p: events.append((k, p)))
    toks = list(range(100, 112))  # 3 full pages
    sb = bm.allocate_prompt(toks, len(toks))
    assert sb is not None and len(sb.pages) == 3 and sb.num_cached_tokens == 0
    bm.commit_full_pages(sb, toks, 12)
    assert events[-1][0] == "BlockStored"
    assert events[-1][1]["block_hashes"] == chain_hashes(toks, 4)
    assert events[-1][1]["token_ids"] == toks
    bm.free(sb)
    assert bm.num_free() == 4
    # same prefix: last page is recomputed (a token must be left to compute)
    sb2 = bm.allocate_prompt(toks, len(toks))
    assert sb2.num_cached_tokens == 8
    bm.free(sb2)
    # a disjoint 4-page prompt forces evictions of the cached pages
    other = list(range(500, 516))
    sb3 = bm.allocate_prompt(other, len(other))
    assert sb3 is not None
    assert any(k == "BlockRemoved" for k, _ in events)


def test_hash_chain_matches_router_definition():
    toks = list(range(40))
    hs = chain_hashes(toks, 16)
    assert len(hs) == 2
    assert hs[0] == hash_chunk(0, toks[:16])
    assert hs[1] == hash_chunk(hs[0], toks[16:32])

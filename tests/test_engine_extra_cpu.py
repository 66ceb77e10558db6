"""More engine behaviour on CPU: stop tokens, min_tokens, abort, seeded
sampling, duplicate ids, the per-sequence prefill chunk cap, the sequence
limit, shared prefix pages and cache clearing."""

import pytest
import torch

from infera_b200.engine.block_manager import BlockManager
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams


def _engine(**kw):
    kw.setdefault("num_pages", 64)
    return LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, **kw), device="cpu")


def _prompt(seed, n=20):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1024, (n,), generator=g).tolist()


def test_stop_token_and_min_tokens():
    eng = _engine()
    p = _prompt(1)
    free = eng.generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0]
    stop = free[2]
    first = free.index(stop)
    out = eng.generate([p], SamplingParams(max_tokens=8, ignore_eos=True, stop_token_ids=[stop]))[0]
    assert out == free[:first + 1]
    # min_tokens defers the stop check
    out = eng.generate([p], SamplingParams(max_tokens=8, ignore_eos=True, stop_token_ids=[stop],
                                           min_tokens=first + 2))[0]
    assert len(out) > first + 1 and out == free[:len(out)]


def test_abort_frees_pages_and_finishes():
    eng = _engine()
    free0 = eng.bm.num_free()
    eng.add_request("a", _prompt(2, 40), SamplingParams(max_tokens=50, ignore_eos=True))
    eng.step()
    assert eng.bm.num_free() < free0
    assert eng.abort_request("a")
    assert not eng.has_unfinished()
    assert not eng.abort_request("a")          # already gone
    with pytest.raises(ValueError):
        eng.add_request("b", [1, 2, 3])
        eng.add_request("b", [1, 2, 3])        # duplicate id


def test_seeded_sampling_is_reproducible():
    eng = _engine()
    p = _prompt(3)
    sp = SamplingParams(max_tokens=6, ignore_eos=True, temperature=1.0, seed=1234)
    a = eng.generate([p], sp)[0]
    b = eng.generate([p], sp)[0]
    c = eng.generate([p], SamplingParams(max_tokens=6, ignore_eos=True, temperature=1.0, seed=99))[0]
    assert a == b and len(a) == 6
    assert a != c   # 6 tokens from a 1024-token vocabulary at temperature 1


def test_long_prefill_cap_and_sequence_limit():
    eng = _engine(max_batched_tokens=256, max_num_seqs=2, long_prefill_threshold=32)
    for i in range(3):
        eng.add_request(f"r{i}", _prompt(10 + i, 100), SamplingParams(max_tokens=2, ignore_eos=True))
    sched = eng.scheduler.schedule()
    assert len(sched.prefills) == 2                      # max_num_seqs
    assert all(c.num_tokens <= 32 for c in sched.prefills)
    for c in sched.prefills:                             # leave the scheduler consistent
        eng.scheduler.abort(c.req.request_id)


def test_shared_prefix_pages_are_refcounted():
    bm = BlockManager(num_pages=8, page_size=4)
    toks = list(range(12))
    a = bm.allocate_prompt(toks + [100], 13)
    bm.commit_full_pages(a, toks + [100], 12)
    b = bm.allocate_prompt(toks + [200], 13)
    assert b.num_cached_tokens == 12 and b.pages[:3] == a.pages[:3]
    bm.free(a)
    # b still holds the shared pages: a new prompt cannot take them
    c = bm.allocate_prompt(list(range(500, 520)), 20)
    assert c is None or not set(c.pages) & set(b.pages)
    bm.free(b)
    if c is not None:
        bm.free(c)
    events = []
    bm.event_sink = lambda k, p: events.append(k)
    bm.clear_cache()
    # every page but the reserved padding page 0 is free again
    assert bm.cached_hashes() == [] and bm.num_free() == 8 - bm.reserved and events == ["AllBlocksCleared"]


def test_mixed_step_prefill_cap_while_decoding():
    """While sequences decode, prompt chunks joining a step are capped (the
    step is their inter-token gap); with nothing decoding, prompts get the
    whole budget. Outputs are unchanged by the chunking."""
    eng = _engine(num_pages=256, max_batched_tokens=256, mixed_prefill_tokens=24)
    eng.add_request("d", _prompt(20, 30), SamplingParams(max_tokens=40, ignore_eos=True))
    eng.step()                                            # "d" prefills, then decodes
    eng.add_request("p", _prompt(21, 200), SamplingParams(max_tokens=3, ignore_eos=True))
    sched = eng.scheduler.schedule()
    assert len(sched.decodes) == 1
    assert sum(c.num_tokens for c in sched.prefills) <= 24
    for c in sched.prefills + sched.decodes:
        eng.scheduler.abort(c.req.request_id)
    eng.requests.clear()
    # nothing decoding: the full budget
    eng.add_request("q", _prompt(22, 200), SamplingParams(max_tokens=3, ignore_eos=True))
    sched = eng.scheduler.schedule()
    assert not sched.decodes and sum(c.num_tokens for c in sched.prefills) == 200
    eng.scheduler.abort("q")
    eng.requests.clear()
    # same tokens as an uncapped engine
    ref = _engine(num_pages=256, max_batched_tokens=256, mixed_prefill_tokens=0)
    ps = [_prompt(30 + i, 90 + 20 * i) for i in range(3)]
    sp = SamplingParams(max_tokens=5, ignore_eos=True)
    assert eng.generate(ps, sp) == ref.generate(ps, sp)


def test_block_manager_keeps_sequences_in_page_runs():
    """A sequence's next page is its last page + 1 when that one is free, so
    pages come in consecutive runs even after other sequences freed theirs."""
    from infera_b200.engine.block_manager import BlockManager

    bm = BlockManager(num_pages=200, page_size=16, enable_prefix_cache=False)
    a = bm.allocate_prompt(list(range(40 * 16)), 40 * 16)
    b = bm.allocate_prompt(list(range(20 * 16)), 20 * 16)
    assert a.pages == list(range(a.pages[0], a.pages[0] + 40))
    bm.free(a)
    c = bm.allocate_prompt(list(range(30 * 16)), 30 * 16)
    assert c.pages == list(range(c.pages[0], c.pages[0] + 30))
    assert bm.ensure_capacity(b, 28 * 16)            # b grows past its run end into free pages
    runs = sum(1 for i in range(1, len(b.pages)) if b.pages[i] != b.pages[i - 1] + 1)
    assert runs <= 1
    free_before = bm.num_free()
    bm.free(b)
    bm.free(c)
    assert bm.num_free() == free_before + 28 + 30 and bm.num_free() == 199
    for _ in range(3000):                            # stale stack entries stay bounded
        s = bm.allocate_prompt(list(range(33)), 33)
        bm.free(s)
    assert len(bm.free_plain) <= 2 * len(bm.free_set) + 1024


def test_block_manager_keeps_tiles_consecutive_under_interleaved_growth():
    """Sequences that grow side by side (decode steps) still fill every
    8-page key tile with one run of consecutive pages: the rest of a tile
    is set aside for its sequence when the tile's first page is taken, and
    returned when the sequence is freed."""
    from infera_b200.engine.block_manager import BlockManager, SeqBlocks

    bm = BlockManager(num_pages=4096, page_size=16, enable_prefix_cache=False)
    seqs = [SeqBlocks() for _ in range(6)]
    free0 = bm.num_free()
    for step in range(1, 40 * 16 + 1):          # 40 pages each, one token at a time, interleaved
        for sb in seqs:
            assert bm.ensure_capacity(sb, step)
    for sb in seqs:
        pages = sb.pages
        assert len(pages) == 40
        for t in range(0, 40, 8):
            assert pages[t:t + 8] == list(range(pages[t], pages[t] + 8))
    for sb in seqs:
        bm.free(sb)
        assert sb.run_ahead == []
    assert bm.num_free() == free0

"""KV tiering on the GPU: a prefix evicted from HBM is saved to the host
tier by the batched gather + copy-out, promoted back asynchronously (loader
thread, side stream, the request parked until the copies land), and the
promoted pages are byte-identical to the ones first computed; the first
token's logits then match a fresh engine that recomputes the prompt."""

import pytest
import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.ops import kernels as K
from infera_b200.utils.hashing import chain_hashes

pytestmark = pytest.mark.gpu


def _engine(**kw):
    cfg = EngineConfig(model="tiny-dense-gpu", num_pages=40, max_num_seqs=4, max_batched_tokens=256,
                       use_cuda_graphs=False, **kw)
    return LLMEngine(cfg, device="cuda:0")


def _pages_of(eng, hashes):
    return [eng.bm.hash_to_page.get(h) for h in hashes]


def _gather(eng, pages):
    idx = torch.tensor(pages, dtype=torch.int32, device="cuda")
    L, _, H = eng.runner.k_cache.shape
    out = torch.empty(len(pages), 2 * L * 16 * H, dtype=torch.bfloat16, device="cuda")
    K.kv_page_copy(eng.runner.k_cache, eng.runner.v_cache, out, idx, 16, gather=True, page_major=True)
    torch.cuda.synchronize()
    return out


def _first_logits(eng, rid, prompt):
    eng.add_request(rid, prompt, SamplingParams(max_tokens=1, ignore_eos=True))
    for _ in range(1000):
        outs = eng.step()
        if any(o.request_id == rid and o.new_token_ids for o in outs):
            return eng.runner.last_logits[0].float().clone()
    raise AssertionError("no token")


@pytest.mark.parametrize("spec", ["host:1", "pinned:1"])
def test_tier_evict_save_and_async_promote_match_recompute(spec):
    """Both host tiers: packed blobs, and the page-locked arena of page slots
    written and read by DMA."""
    g = torch.Generator().manual_seed(11)
    a = torch.randint(0, 4000, (320,), generator=g).tolist()          # 20 full pages
    eng = _engine(kv_tier=spec)
    sp = SamplingParams(max_tokens=2, ignore_eos=True)
    eng.generate([a], sp)
    hashes = chain_hashes(a, 16)[:19]
    before = _gather(eng, _pages_of(eng, hashes))
    for _ in range(3):                     # other prompts push A's pages out of HBM
        eng.generate([torch.randint(0, 4000, (300,), generator=g).tolist()], sp)
    eng.tier.flush()
    assert all(p is None for p in _pages_of(eng, hashes[:4])), "A's head pages should be evicted"
    assert eng.tier.stats["saved"] >= 19 and eng.tier.stats["save_batches"] >= 1
    a2 = a + [7, 8, 9]
    got = _first_logits(eng, "a2", a2)
    assert eng.tier.stats["loads"] >= 1 and eng.bm.stats["tier_hit_tokens"] >= 16 * 4
    after = _gather(eng, _pages_of(eng, hashes))
    assert torch.equal(after, before)      # promoted pages are the pages first computed
    assert K.scratch(torch.device("cuda", 0)).read_status() == 0
    ref = _first_logits(_engine(), "r", a2)
    err = float((got - ref).norm() / ref.norm())
    assert err < 2e-2, err
    eng.tier.close()


def test_tier_promote_from_kvd_shared_arena_by_dma(tmp_path):
    """With the kvd daemon's shared arena (handed over SCM_RIGHTS) page-locked
    by cudaHostRegister, promotes copy each page straight from the arena
    into device memory; the pages come back byte-identical."""
    import asyncio
    import threading

    from infera_b200.kvd.server import KvdServer
    from infera_b200.kvd.shared_arena import SharedArena
    from infera_b200.kvd.store import HostStore

    path = str(tmp_path / "kvd.sock")
    store = HostStore(0, arena=SharedArena(256, 1 << 16))
    loop = asyncio.new_event_loop()
    ready = threading.Event()

    async def serve():
        srv = KvdServer(path, store)
        await srv.start()
        ready.set()

    th = threading.Thread(target=lambda: (loop.run_until_complete(serve()), loop.run_forever()), daemon=True)
    th.start()
    assert ready.wait(10)
    try:
        g = torch.Generator().manual_seed(12)
        a = torch.randint(0, 4000, (320,), generator=g).tolist()
        eng = _engine(kv_tier=f"kvd:{path}")
        assert eng.tier.arena_t is not None                  # the arena is page-locked for DMA
        sp = SamplingParams(max_tokens=2, ignore_eos=True)
        eng.generate([a], sp)
        hashes = chain_hashes(a, 16)[:19]
        before = _gather(eng, _pages_of(eng, hashes))
        for _ in range(3):
            eng.generate([torch.randint(0, 4000, (300,), generator=g).tolist()], sp)
        eng.tier.flush()
        _first_logits(eng, "a2", a + [1, 2])
        assert eng.tier.stats["direct_pages"] >= 16, eng.tier.stats
        after = _gather(eng, _pages_of(eng, hashes))
        assert torch.equal(after, before)
        assert K.scratch(torch.device("cuda", 0)).read_status() == 0
        eng.tier.close()
    finally:
        loop.call_soon_threadsafe(loop.stop)

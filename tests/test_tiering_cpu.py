"""KV chunk format v2, page gather/scatter, and engine tiering: a prefix
evicted from HBM is saved to the host tier and promoted back on the next
request, with outputs unchanged."""

import pytest
import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.packed_format import ChunkHeader, PackedFormatError, pack_chunk, unpack_chunk
from infera_b200.engine.request import SamplingParams
from infera_b200.models.reference import reference_greedy
from infera_b200.ops import kernels as K


def test_packed_format_roundtrip_and_alignment():
    h = ChunkHeader(chunk_tokens=16, block_size=16, num_layers=3, hidden_dim=64, dtype="bf16",
                    layer_names=("a", "b", "c"))
    payload = bytes(range(256)) * (h.payload_bytes // 256)
    blob = pack_chunk(h, payload)
    h2, p2 = unpack_chunk(blob)
    assert h2.payload_byte_offset % 4096 == 0 and bytes(p2) == payload and h2.layer_names == ("a", "b", "c")
    with pytest.raises(PackedFormatError):
        unpack_chunk(blob[:100])
    with pytest.raises(PackedFormatError):
        pack_chunk(h, payload[:-2])


def test_kv_page_copy_roundtrip():
    L, slots, H = 2, 64, 32
    k = torch.randn(L, slots, H).to(torch.bfloat16)
    v = torch.randn(L, slots, H).to(torch.bfloat16)
    pages = torch.tensor([3, 1], dtype=torch.int32)
    chunk = torch.empty(2 * L * 32 * H, dtype=torch.bfloat16)
    K.kv_page_copy(k, v, chunk, pages, gather=True)
    c = chunk.view(2, L, 32, H)
    assert torch.equal(c[0, 1, :16], k[1, 48:64]) and torch.equal(c[1, 0, 16:], v[0, 16:32])
    k2, v2 = torch.zeros_like(k), torch.zeros_like(v)
    K.kv_page_copy(k2, v2, chunk, pages, gather=False)
    assert torch.equal(k2[:, 48:64], k[:, 48:64]) and torch.equal(v2[:, 16:32], v[:, 16:32])


@pytest.mark.parametrize("async_load,spec", [(True, "host:0.05"), (False, "host:0.05"), (True, "pinned:0.05"),
                                              (False, "pinned:0.05")])
def test_engine_tier_save_and_promote(async_load, spec):
    """Asynchronous promote: the request waits (parked) while the loader
    copies its prefix in, the engine keeps stepping; inline promote: the
    copies are issued at admission. Both host tiers: packed blobs, and the
    arena of page slots written and read by copy."""
    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=12, max_batched_tokens=256,
                                 kv_tier=spec, kv_tier_async=async_load), device="cpu")
    g = torch.Generator().manual_seed(4)
    a = torch.randint(0, 1000, (64,), generator=g).tolist()
    sp = SamplingParams(max_tokens=2, ignore_eos=True)
    eng.generate([a], sp)
    for _ in range(3):  # other prompts push A's pages out of HBM
        eng.generate([torch.randint(0, 1000, (64,), generator=g).tolist()], sp)
    eng.tier.flush()
    assert eng.tier.stats["saved"] >= 4
    a2 = a + [5, 6, 7]
    out = eng.generate([a2], SamplingParams(max_tokens=3, ignore_eos=True))[0]
    assert eng.bm.stats["tier_hit_tokens"] >= 48
    ref, margins = reference_greedy(eng.model, a2, 3)
    for i, (x, y) in enumerate(zip(out, ref)):
        if x != y:
            assert margins[i] < 0.05
            break


def test_tier_promote_abort_releases_pages_after_landing():
    """A request aborted while its promote is in flight keeps its pages until
    the copies land (they are being written), then frees them."""
    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=12, max_batched_tokens=256,
                                 kv_tier="host:0.05"), device="cpu")
    g = torch.Generator().manual_seed(9)
    a = torch.randint(0, 1000, (64,), generator=g).tolist()
    sp = SamplingParams(max_tokens=2, ignore_eos=True)
    eng.generate([a], sp)
    for _ in range(3):
        eng.generate([torch.randint(0, 1000, (64,), generator=g).tolist()], sp)
    eng.tier.flush()
    free0 = eng.bm.num_free()
    eng.add_request("x", a + [1, 2], SamplingParams(max_tokens=4, ignore_eos=True))
    eng.step()                                    # admitted and parked while the promote runs
    assert "x" in eng.scheduler.loading
    assert eng.abort_request("x")
    assert "x" in eng.scheduler.loading           # pages held until the copies land
    for _ in range(200):
        if not eng.has_unfinished():
            break
        eng.step()
    assert not eng.scheduler.loading and eng.bm.num_free() == free0


def test_engine_tier_file_per_chunk_l3_under_reaper_budget(tmp_path, monkeypatch):
    """kv_tier host:<tiny>:files:<dir>: evicted pages spill from the host
    store to one file per chunk; the reaper keeps the directory under its
    budget; a promote of a reaped chunk misses instead of failing."""
    d = tmp_path / "l3"
    page_bytes = 2 * 2 * 16 * 2 * 64 * 2 + 8192          # tiny-dense page payload + header, rounded up
    monkeypatch.setenv("INFERA_KVD_L3_BUDGET_BYTES", str(6 * page_bytes))
    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=12, max_batched_tokens=256,
                                 kv_tier=f"host:0.0001:files:{d}"), device="cpu")
    g = torch.Generator().manual_seed(6)
    sp = SamplingParams(max_tokens=2, ignore_eos=True)
    for _ in range(6):
        eng.generate([torch.randint(0, 1000, (64,), generator=g).tolist()], sp)
    eng.tier.flush()
    files = [p for p in d.iterdir() if p.name.endswith(".kvcache")]
    assert files and sum(p.stat().st_size for p in files) <= 6 * page_bytes
    l3 = eng.tier.store.l3
    assert l3.reaper.stats["reaped_files"] > 0 and len(files) <= len(l3.index) + 1


def test_tier_ttft_bench_cpu(capsys):
    """The tier-hit vs recompute TTFT bench: with the HBM pool capped below
    three prefixes, session 0 comes back from the host tier."""
    import json

    from infera_b200.bench.tier_ttft import main

    main(["--model", "tiny-dense", "--prefix", "400", "--increment", "16", "--sessions", "3", "--hbm-kv-gb",
          "0.002", "--host-gb", "1", "--max-batched-tokens", "256", "--device", "cpu"])
    d = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert d["tier_loads"] >= 1 and d["tier_hit_cached_tokens"] >= 384
    assert d["hbm_hit_cached_tokens"] >= 384 and len(d["ttft_cold_s"]) == 3


def test_pinned_store_lru_pins_and_listeners():
    from infera_b200.engine.pinned_store import PinnedPageStore

    st = PinnedPageStore(capacity_bytes=3 * 64)
    st.bind(32, torch.bfloat16, pin=False)                 # 64-byte pages: 3 slots
    dropped = []
    st.add_listener(lambda k, spilled: dropped.append(k))
    a = st.reserve([b"a", b"b", b"c"])
    assert sorted(a) == [0, 1, 2] and not st.exists(b"a")  # reserved: invisible
    assert st.commit([b"a", b"b", b"c"]) == [b"a", b"b", b"c"]
    assert st.reserve([b"a"]) == [None]                    # already held
    pinned = st.acquire([b"a"])                            # a is read: refreshed and pinned
    assert st.reserve([b"d"]) != [-1] and dropped == [b"b"]
    st.commit([b"d"])
    st.reserve([b"e"])                                     # c goes (a is pinned)
    assert dropped == [b"b", b"c"]
    st.commit([b"e"])
    assert st.reserve([b"f"]) != [-1] and dropped[-1] == b"d"  # a is the oldest but pinned: d goes
    st.release(pinned)
    assert st.exists_many([b"a", b"d", b"e"]) == [True, False, True]

"""Host-side launch planning of the kernels (no GPU needed): prefill tile
lists, key-share counts, MLA split counts and GEMM plans."""

import pytest

from infera_b200.ops import _native
from infera_b200.ops import kernels as K


def _lib_or_skip():
    try:
        return _native.kernels()
    except Exception as e:  # the library is built by the build step
        pytest.skip(f"kernel library not built: {e}")


def test_prefill_tiles_two_tile_items_cover_every_block_longest_first():
    q_lens = [1, 300, 1000, 128]
    items = K.prefill_tiles(q_lens, 256)
    covered = {(s, qb + d) for s, qb in items for d in (0, 1)}
    for s, n in enumerate(q_lens):
        for b in range((n + 127) // 128):
            assert (s, b) in covered
        assert all(qb % 2 == 0 for seq, qb in items if seq == s)
    assert [qb for _, qb in items] == sorted((qb for _, qb in items), reverse=True)
    one = K.prefill_tiles(q_lens, 128)
    assert sorted(one) == sorted((s, b) for s, n in enumerate(q_lens) for b in range((n + 127) // 128))


def test_prefill_key_shares_only_for_short_chunks_over_long_contexts():
    # 128 two-tile CTAs (1024 queries x 32 heads) are not split (measured slower)
    assert K.prefill_kv_splits(32, 4, 8192) == 1
    # 32 CTAs (one 224-query chunk) over 8192 keys: 4 shares measured best
    assert K.prefill_kv_splits(32, 1, 8192) == 4
    # short contexts and full waves are never split
    assert K.prefill_kv_splits(32, 1, 1024) == 1
    assert K.prefill_kv_splits(64, 4, 32768) == 1
    for heads, tiles, ctx in [(8, 1, 32768), (32, 2, 16384), (16, 3, 65536)]:
        sp = K.prefill_kv_splits(heads, tiles, ctx)
        assert 1 <= sp <= 16 and -(-ctx // 128) // sp >= 4


def test_mla_split_counts_for_128_key_tiles():
    _lib_or_skip()
    from infera_b200.ops import mla as M

    if M.mla_key_tile() != 128:
        pytest.skip("32-key MLA tiles selected")
    assert M.mla_splits(64, 4096) == 1       # 128 CTAs already fill one wave
    assert M.mla_splits(16, 4096) == 4       # 32 CTAs: four shares of 8 tiles
    assert M.mla_splits(1, 4096) == 32       # one query: one tile per share
    assert M.mla_splits(64, 300) == 1


def test_gemm_plans():
    _lib_or_skip()
    p = K.gemm_plan(0, 4096, 4096)           # an empty token set plans without dividing by zero
    assert p["q_tiles"] >= 1
    p = K.gemm_plan(64, 28672, 4096)         # decode gate/up: swap-AB, stream-K
    assert p["swap"] == 1 and p["bn"] == 64 and p["splits"] == -1
    p = K.gemm_plan(288, 28672, 4096)        # mixed step, wide weights: two token tiles per weight tile
    assert p["swap"] == 1 and p["q_tiles"] == 2 and p["bn"] == 144
    p = K.gemm_plan(288, 4096, 14336)        # mixed step, narrow weights: token rows on the MMA's M side
    assert p["swap"] == 0 and p["bn"] == 256
    p = K.gemm_plan(8, 4096, 4096)           # decode o-projection: split K over too few tiles
    assert p["swap"] == 1 and p["splits"] > 1

"""tcgen05 paged decode attention against the fp32 oracle, including split
KV, multiple GQA group sizes, block-table row indirection and sequences
whose last tile is partial."""

import math

import pytest
import torch

from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-6))


def _setup(lens, hkv, D=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    pages = sum((n + 15) // 16 for n in lens) + 3
    perm = torch.randperm(pages, generator=g)
    width = max((n + 15) // 16 for n in lens) + 2
    bt = torch.zeros(len(lens) + 2, width, dtype=torch.int32)
    rows = list(range(len(lens) + 2))[2:] + [0, 1]
    rows = rows[: len(lens)]
    k = 0
    for i, n in enumerate(lens):
        for j in range((n + 15) // 16):
            bt[rows[i], j] = perm[k]
            k += 1
    kc = torch.randn(pages * 16, hkv * D, generator=g).to(torch.bfloat16)
    vc = torch.randn(pages * 16, hkv * D, generator=g).to(torch.bfloat16)
    return kc, vc, bt, torch.tensor(rows, dtype=torch.int32)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 2), (8, 8), (64, 8)])
@pytest.mark.parametrize("lens,splits", [([1, 17, 128, 129, 300], 1), ([2000, 5, 8191], 5), ([33] * 20, 3)])
def test_decode_tc(hq, hkv, lens, splits):
    kc, vc, bt, rows = _setup(lens, hkv, seed=len(lens) + hq)
    q = torch.randn(len(lens), (hq + 2 * hkv) * 128).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(128)
    ref = K.attn_decode(q, kc, vc, bt, sl, hq, hkv, scale, bt_rows=rows)
    out = K.attn_decode(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), sl.cuda(), hq, hkv, scale, splits=splits,
                        bt_rows=rows.cuda(), impl="tc")
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    assert _rel(out.cpu(), ref) < 2e-2


@pytest.mark.parametrize("lens,splits", [([1000, 129, 2048], 1), ([5000, 77], 4)])
def test_decode_tc_consecutive_pages(lens, splits):
    """Eight consecutive pages load as one 128-row box per half; runs that
    start mid-tile, partial last tiles and a break inside a tile take the
    page-by-page path."""
    hq, hkv = 32, 8
    g = torch.Generator().manual_seed(21)
    width = max((n + 15) // 16 for n in lens) + 2
    pages = len(lens) * width + 8
    bt = torch.zeros(len(lens), width, dtype=torch.int32)
    start = 3
    for i, n in enumerate(lens):
        np_ = (n + 15) // 16
        bt[i, :np_] = torch.arange(start, start + np_, dtype=torch.int32)
        start += np_ + 1
    bt[0, 10] = pages - 1          # one page out of line inside the first sequence's second tile
    kc = torch.randn(pages * 16, hkv * 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(pages * 16, hkv * 128, generator=g).to(torch.bfloat16)
    q = torch.randn(len(lens), (hq + 2 * hkv) * 128, generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(128)
    ref = K.attn_decode(q, kc, vc, bt, sl, hq, hkv, scale)
    out = K.attn_decode(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), sl.cuda(), hq, hkv, scale, splits=splits,
                        impl="tc")
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    assert _rel(out.cpu(), ref) < 2e-2

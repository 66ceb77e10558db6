"""Numerics of every sm_100a kernel against the fp32 PyTorch oracle of the
same op (the CPU path of :mod:`infera_b200.ops.kernels`)."""

import math

import pytest
import torch

from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-6))


def _check_status():
    st = K.scratch(torch.device(DEV, 0)).read_status()
    assert st == 0, f"kernel status {st}"


@pytest.mark.parametrize("M,N,K_", [
    (1, 4096, 4096), (7, 6144, 4096), (16, 1024, 512), (64, 4096, 14336), (128, 28672, 4096),
    (129, 4096, 4096), (256, 6144, 4096), (1000, 4096, 4096), (2048, 1024, 4096), (300, 520, 192),
])
def test_gemm_bf16(M, N, K_):
    torch.manual_seed(0)
    x = (torch.randn(M, K_, device=DEV) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K_, device=DEV) / math.sqrt(K_)).to(torch.bfloat16)
    y = K.linear(x, w)
    torch.cuda.synchronize()
    _check_status()
    ref = K.linear(x.cpu(), w.cpu())
    assert _rel_err(y.cpu(), ref) < 1e-2


@pytest.mark.parametrize("force_split", [1, 3])
@pytest.mark.parametrize("M", [5, 200])
def test_gemm_swiglu(M, force_split):
    torch.manual_seed(1)
    N, K_ = 2048, 1024
    x = (torch.randn(M, K_, device=DEV)).to(torch.bfloat16)
    w = (torch.randn(N, K_, device=DEV) / math.sqrt(K_)).to(torch.bfloat16)
    y = K.linear(x, w, swiglu=True, force_split=force_split)
    torch.cuda.synchronize()
    _check_status()
    ref = K.linear(x.cpu(), w.cpu(), swiglu=True)
    assert y.shape == (M, N // 2)
    assert _rel_err(y.cpu(), ref) < 1e-2
    # workspace is left zeroed for the next split-K call
    assert float(K.scratch().gemm_ws.abs().sum()) == 0.0


@pytest.mark.parametrize("M,N,K_,swiglu", [(1, 28672, 4096, True), (64, 28672, 4096, True),
                                            (64, 28672, 4096, False), (128, 28672, 4096, False),
                                            (288, 28672, 4096, True), (3840, 2560, 1024, False)])
def test_gemm_stream_k(M, N, K_, swiglu):
    """More tiles than SMs but a poor last wave: whole tiles for the full
    waves, the rest shared out k-step by k-step; partial tiles meet in the
    fp32 workspace, which is left zeroed, as are the per-tile counters of the
    in-kernel reduction (288 x 28672: swap-AB with 296 whole tiles; 3840 x
    2560: token-row tiles with 120 whole tiles)."""
    torch.manual_seed(4)
    assert K.gemm_plan(M, N, K_)["splits"] == -1
    x = (torch.randn(M, K_, device=DEV) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K_, device=DEV) / math.sqrt(K_)).to(torch.bfloat16)
    y = K.linear(x, w, swiglu=swiglu)
    torch.cuda.synchronize()
    _check_status()
    ref = K.linear(x.cpu(), w.cpu(), swiglu=swiglu)
    assert _rel_err(y.cpu(), ref) < 1e-2
    assert float(K.scratch().gemm_ws.abs().sum()) == 0.0
    sc = K.scratch()
    if sc.gemm_ctr.numel():
        assert int(sc.gemm_ctr.abs().sum()) == 0


def test_gemm_repeated_split_consistent():
    torch.manual_seed(2)
    x = torch.randn(8, 4096, device=DEV).to(torch.bfloat16)
    w = (torch.randn(4096, 4096, device=DEV) / 64).to(torch.bfloat16)
    a = K.linear(x, w)
    b = K.linear(x, w)
    torch.cuda.synchronize()
    assert _rel_err(a, b) < 1e-3


@pytest.mark.parametrize("H", [4096, 8192, 5120])
def test_rmsnorm_and_add(H):
    torch.manual_seed(3)
    T = 37
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    d = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    w = torch.randn(H, device=DEV).to(torch.bfloat16)
    y = K.rmsnorm(x, w, 1e-5)
    ref = K.rmsnorm(x.cpu(), w.cpu(), 1e-5)
    assert _rel_err(y.cpu(), ref) < 1e-2
    r_gpu = x.clone()
    r_cpu = x.cpu().clone()
    y2 = K.add_rmsnorm(d, r_gpu, w, 1e-5)
    ref2 = K.add_rmsnorm(d.cpu(), r_cpu, w.cpu(), 1e-5)
    torch.cuda.synchronize()
    assert _rel_err(r_gpu.cpu(), r_cpu) < 1e-2
    assert _rel_err(y2.cpu(), ref2) < 1e-2


def test_rope_kvwrite():
    torch.manual_seed(4)
    T, hq, hkv, D = 19, 32, 8, 128
    cs = K.rope_cos_sin(4096, D, 500000.0, {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                              "original_max_position_embeddings": 8192})
    qkv = torch.randn(T, (hq + 2 * hkv) * D).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32)
    slots = torch.randperm(64, dtype=torch.int32)[:T]
    slots[3] = -1
    kc = torch.zeros(64, hkv * D, dtype=torch.bfloat16)
    vc = torch.zeros(64, hkv * D, dtype=torch.bfloat16)
    qkv_g, kc_g, vc_g = qkv.cuda(), kc.cuda(), vc.cuda()
    K.rope_kvwrite(qkv_g, pos.cuda(), slots.cuda(), cs.cuda(), hq, hkv, D, kc_g, vc_g)
    K.rope_kvwrite(qkv, pos, slots, cs, hq, hkv, D, kc, vc)
    torch.cuda.synchronize()
    assert _rel_err(qkv_g.cpu(), qkv) < 1e-2
    assert _rel_err(kc_g.cpu(), kc) < 1e-2
    assert torch.equal(vc_g.cpu(), vc)


def test_embed_and_sample():
    torch.manual_seed(5)
    table = torch.randn(1000, 256).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (9,), dtype=torch.int32)
    e = K.embed(ids.cuda(), table.cuda())
    assert torch.equal(e.cpu(), table[ids.long()])
    logits = torch.randn(6, 128256).to(torch.bfloat16)
    g = K.sample(logits.cuda())
    assert torch.equal(g.cpu(), torch.argmax(logits.float(), -1).to(torch.int32))
    temp = torch.tensor([0.0, 1.0, 0.7, 1.0, 0.0, 2.0])
    seeds = torch.tensor([1, 2, 3, 4, 5, 6], dtype=torch.int64)
    small = logits[:, :512].contiguous()
    s_gpu = K.sample(small.cuda(), temp.cuda(), seeds.cuda())
    s_cpu = K.sample(small, temp, seeds)
    torch.cuda.synchronize()
    assert torch.equal(s_gpu.cpu(), s_cpu)


def _paged_setup(lens, hkv=8, D=128, page=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    n_pages = sum((n + page - 1) // page for n in lens) + 3
    perm = torch.randperm(n_pages, generator=g)
    max_pages = max((n + page - 1) // page for n in lens)
    bt = torch.zeros(len(lens), max_pages, dtype=torch.int32)
    k = 0
    for i, n in enumerate(lens):
        for j in range((n + page - 1) // page):
            bt[i, j] = perm[k]
            k += 1
    kc = (torch.randn(n_pages * page, hkv * D, generator=g)).to(torch.bfloat16)
    vc = (torch.randn(n_pages * page, hkv * D, generator=g)).to(torch.bfloat16)
    return kc, vc, bt


@pytest.mark.parametrize("lens,splits", [([1, 17, 64, 300], 1), ([1, 17, 64, 300], 4), ([5000], 16),
                                         ([33] * 40, 2)])
def test_attn_decode(lens, splits):
    hq, hkv, D = 32, 8, 128
    kc, vc, bt = _paged_setup(lens, hkv, D)
    q = torch.randn(len(lens), (hq + 2 * hkv) * D).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    ref = K.attn_decode(q, kc, vc, bt, sl, hq, hkv, scale)
    out = K.attn_decode(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), sl.cuda(), hq, hkv, scale, splits=splits)
    torch.cuda.synchronize()
    assert _rel_err(out.cpu(), ref) < 2e-2


@pytest.mark.parametrize("q_lens,ctx_lens", [
    ([128], [128]), ([1, 77, 200], [1, 77, 500]), ([300, 5], [1300, 900]), ([1024], [4096 + 1024]),
])
def test_attn_prefill(q_lens, ctx_lens):
    hq, hkv, D = 32, 8, 128
    kc, vc, bt = _paged_setup(ctx_lens, hkv, D, seed=7)
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * D).to(torch.bfloat16)
    q_start = torch.tensor([sum(q_lens[:i]) for i in range(len(q_lens))], dtype=torch.int32)
    ql = torch.tensor(q_lens, dtype=torch.int32)
    cl = torch.tensor(ctx_lens, dtype=torch.int32)
    tiles = torch.tensor(K.prefill_tiles(q_lens), dtype=torch.int32).view(-1, 2)
    scale = 1 / math.sqrt(D)
    ref = K.attn_prefill(q, kc, vc, bt, q_start, ql, cl, tiles, hq, hkv, scale)
    out = K.attn_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), q_start.cuda(), ql.cuda(), cl.cuda(),
                         tiles.cuda(), hq, hkv, scale)
    torch.cuda.synchronize()
    _check_status()
    assert _rel_err(out.cpu(), ref) < 2e-2


@pytest.mark.parametrize("q_lens,ctx_lens,splits", [
    ([200], [8192], 4), ([1, 77, 300], [3000, 77, 2600], 3), ([256, 128], [6000, 6000], 16), ([130], [130], 2),
])
def test_attn_prefill_key_split(q_lens, ctx_lens, splits):
    """Key shares of each query tile over several CTAs, merged by the
    combine kernel: later shares hold rows whose keys are all masked (the
    chunk's first rows see only the early keys) and shares past a short
    sequence's keys are empty."""
    hq, hkv, D = 32, 8, 128
    kc, vc, bt = _paged_setup(ctx_lens, hkv, D, seed=9)
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * D).to(torch.bfloat16)
    q_start = torch.tensor([sum(q_lens[:i]) for i in range(len(q_lens))], dtype=torch.int32)
    ql = torch.tensor(q_lens, dtype=torch.int32)
    cl = torch.tensor(ctx_lens, dtype=torch.int32)
    tiles = torch.tensor(K.prefill_tiles(q_lens), dtype=torch.int32).view(-1, 2)
    scale = 1 / math.sqrt(D)
    ref = K.attn_prefill(q, kc, vc, bt, q_start, ql, cl, tiles, hq, hkv, scale)
    out = K.attn_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), q_start.cuda(), ql.cuda(), cl.cuda(),
                         tiles.cuda(), hq, hkv, scale, kv_splits=splits)
    torch.cuda.synchronize()
    _check_status()
    assert _rel_err(out.cpu(), ref) < 2e-2
    assert K.prefill_kv_splits(hq, tiles.shape[0], max(ctx_lens)) >= 1


@pytest.mark.parametrize("q_lens,ctx_lens", [([300, 1000], [2300, 1000]), ([129], [129])])
def test_attn_prefill_consecutive_pages(q_lens, ctx_lens):
    """Eight consecutive pages load as one 128-row box per 64-dim block; a
    page out of line and partial last tiles take the page-by-page path."""
    hq, hkv, D = 32, 8, 128
    g = torch.Generator().manual_seed(13)
    width = max((n + 15) // 16 for n in ctx_lens)
    n_pages = len(ctx_lens) * (width + 1) + 4
    bt = torch.zeros(len(ctx_lens), width, dtype=torch.int32)
    start = 2
    for i, n in enumerate(ctx_lens):
        npg = (n + 15) // 16
        bt[i, :npg] = torch.arange(start, start + npg, dtype=torch.int32)
        start += npg + 1
    if (ctx_lens[0] + 15) // 16 > 9:
        bt[0, 9] = n_pages - 1         # one page out of line in the first sequence's second tile
    kc = torch.randn(n_pages * 16, hkv * D, generator=g).to(torch.bfloat16)
    vc = torch.randn(n_pages * 16, hkv * D, generator=g).to(torch.bfloat16)
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * D, generator=g).to(torch.bfloat16)
    q_start = torch.tensor([sum(q_lens[:i]) for i in range(len(q_lens))], dtype=torch.int32)
    ql = torch.tensor(q_lens, dtype=torch.int32)
    cl = torch.tensor(ctx_lens, dtype=torch.int32)
    tiles = torch.tensor(K.prefill_tiles(q_lens), dtype=torch.int32).view(-1, 2)
    scale = 1 / math.sqrt(D)
    ref = K.attn_prefill(q, kc, vc, bt, q_start, ql, cl, tiles, hq, hkv, scale)
    out = K.attn_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), q_start.cuda(), ql.cuda(), cl.cuda(),
                         tiles.cuda(), hq, hkv, scale)
    torch.cuda.synchronize()
    _check_status()
    assert _rel_err(out.cpu(), ref) < 2e-2


def test_attn_prefill_divergent_rescale():
    """Rows whose running max grows by different amounts across KV tiles, so
    the lazy O rescale is needed by some rows of a warp and not others."""
    hq, hkv, D = 32, 8, 128
    ctx = 1024
    kc, vc, bt = _paged_setup([ctx], hkv, D, seed=11)
    growth = torch.linspace(0.2, 4.0, kc.shape[0])[:, None]
    kc = (kc.float() * growth).to(torch.bfloat16)
    q = torch.randn(ctx, (hq + 2 * hkv) * D)
    q[:, : hq * D] *= (torch.arange(ctx) % 7 + 1).float()[:, None] * 0.5
    q = q.to(torch.bfloat16)
    q_start = torch.tensor([0], dtype=torch.int32)
    ql = torch.tensor([ctx], dtype=torch.int32)
    cl = torch.tensor([ctx], dtype=torch.int32)
    tiles = torch.tensor(K.prefill_tiles([ctx]), dtype=torch.int32).view(-1, 2)
    scale = 1 / math.sqrt(D)
    ref = K.attn_prefill(q, kc, vc, bt, q_start, ql, cl, tiles, hq, hkv, scale)
    out = K.attn_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), q_start.cuda(), ql.cuda(), cl.cuda(),
                         tiles.cuda(), hq, hkv, scale)
    torch.cuda.synchronize()
    _check_status()
    assert _rel_err(out.cpu(), ref) < 2e-2


@pytest.mark.parametrize("M", [8, 64, 288])
def test_deferred_gemm_consumers_match_finalized(M):
    """A split GEMM left in its fp32 workspace, read by add_rmsnorm_ws /
    rope_kvwrite_ws, gives the same rows as the finalized GEMM followed by
    add_rmsnorm / rope_kvwrite, and the workspace is left zeroed."""
    torch.manual_seed(7)
    K._DEFER, was = True, K._DEFER
    try:
        _deferred_case(M)
    finally:
        K._DEFER = was


def _deferred_case(M):
    H, hq, hkv, D = 4096, 32, 8, 128
    x = (torch.randn(M, H, device=DEV) * 0.5).to(torch.bfloat16)
    wo = (torch.randn(H, H, device=DEV) / 64).to(torch.bfloat16)
    nw = torch.randn(H, device=DEV).to(torch.bfloat16)
    h0 = torch.randn(M, H, device=DEV).to(torch.bfloat16)
    assert K._gemm_ws(M, H, H)            # this shape splits
    o = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
    h1, h2 = h0.clone(), h0.clone()
    out1 = K.add_rmsnorm(K.linear(x, wo), h1, nw, 1e-5)
    ws = K.linear_deferred(x, wo, o)
    assert ws is not None
    out2 = K.add_rmsnorm_ws(ws, h2, nw, 1e-5, out=torch.empty_like(h2))
    torch.cuda.synchronize()
    _check_status()
    # same rounding on both paths; only the split partials' atomic order differs
    assert _rel_err(h1.float(), h2.float()) < 1e-3
    assert _rel_err(out1.float(), out2.float()) < 1e-3
    assert float(K.scratch().gemm_ws.abs().sum()) == 0.0
    # qkv -> rope + KV write
    N = (hq + 2 * hkv) * D
    wq = (torch.randn(N, H, device=DEV) / 64).to(torch.bfloat16)
    cos_sin = K.rope_cos_sin(4096, D, 500000.0, device=DEV)
    pos = torch.randint(0, 4000, (M,), device=DEV, dtype=torch.int32)
    slots = torch.randperm(4 * M, device=DEV)[:M].to(torch.int32)
    kc1 = torch.zeros(4 * M, hkv * D, dtype=torch.bfloat16, device=DEV)
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    q1 = K.linear(x, wq)
    K.rope_kvwrite(q1, pos, slots, cos_sin, hq, hkv, D, kc1, vc1)
    q2 = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ws = K.linear_deferred(x, wq, q2)
    if ws is not None:
        K.rope_kvwrite_ws(ws, q2, pos, slots, cos_sin, hq, hkv, D, kc2, vc2)
    else:
        K.rope_kvwrite(q2, pos, slots, cos_sin, hq, hkv, D, kc2, vc2)
    torch.cuda.synchronize()
    _check_status()
    assert _rel_err(q1[:, :hq * D].float(), q2[:, :hq * D].float()) < 1e-3
    assert _rel_err(kc1.float(), kc2.float()) < 1e-3
    assert _rel_err(vc1.float(), vc2.float()) < 1e-3
    assert float(K.scratch().gemm_ws.abs().sum()) == 0.0

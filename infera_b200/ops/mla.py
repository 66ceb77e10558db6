"""Multi-head latent attention ops (DeepSeek-V3 MLA, absorbed form).

* :func:`mla_rope_kvwrite` - RMS-normalise the compressed KV, rotate the
  shared rope key and every head's rope query, write the 576-wide latent
  row of each token into its cache slot (``ib_mla_rope_kvwrite``);
* :func:`mla_attention` - multi-query attention of the absorbed queries
  [nq, hq, 576] over the paged latent cache, values = the first 512 dims of
  each cached row (``ib_mla_decode``, tcgen05); split over the keys when
  few queries are in flight, merged by log-sum-exp;
* :func:`mla_prefill` - prompt chunks NOT absorbed: the latent rows of each
  sequence's context are gathered, up-projected once to per-head
  [k_nope | v] by one GEMM, and the tcgen05 flash-attention kernel scores
  192 dims per head (128 nope + the shared 64-dim rope key read straight
  from the gathered latent rows) and accumulates 128-dim values
  (``ib_attn_prefill_ext``). Per query-key pair that is 320 MACs per head
  instead of the absorbed form's 1088, and the output needs no W_UV
  absorption.

On CPU both run the same math in PyTorch (fp32).
"""

from __future__ import annotations

import math

import torch

from infera_b200.ops import _native
from infera_b200.ops import kernels as K

DL, DR = 512, 64
DQK = DL + DR
PAGE = 16


def mla_key_tile() -> int:
    """Keys per tile of the decode kernel (128, or 32 with INFERA_MLA_TILE=32)."""
    try:
        return int(_native.kernels().ib_mla_key_tile())
    except Exception:
        return 128


def mla_splits(nq: int, max_kvlen: int, num_sms: int = 148) -> int:
    """Key splits per query. 32-key tiles: enough CTAs (nq x 2 value halves
    x splits) to cover the SMs, each split keeping at least 4 tiles.
    128-key tiles (one CTA per SM): the split count that minimises the
    work on the busiest SM, waves x (tiles per split + one tile's worth of
    per-CTA start-up: the resident query load and the pipeline fill),
    fewest splits on a tie."""
    bt = mla_key_tile()
    tiles = max(1, -(-max_kvlen // bt))
    if bt == 32:
        want = max(1, -(-num_sms // (2 * max(nq, 1))))
        return max(1, min(want, tiles // 4 if tiles >= 8 else 1, 64))
    ctas = 2 * max(nq, 1)
    best, best_cost = 1, None
    for sp in range(1, min(64, tiles) + 1):
        cost = -(-ctas * sp // num_sms) * (-(-tiles // sp) + 1)
        if best_cost is None or cost < best_cost:
            best, best_cost = sp, cost
    return best


def mla_rope_kvwrite(q: torch.Tensor, kva: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor,
                     cos_sin: torch.Tensor, norm_w: torch.Tensor, eps: float, cache: torch.Tensor) -> None:
    """q [T, hq, 576] (rope part rotated in place), kva [T, 576] (the
    kv_a projection: compressed KV then the raw rope key), cache [slots, 576]."""
    T, hq, _ = q.shape
    if not q.is_cuda:
        dr = cos_sin.shape[1] * 2
        dl = kva.shape[1] - dr
        half = dr // 2
        cs = cos_sin[pos.long()]                       # [T, 32, 2]
        c, s = cs[..., 0], cs[..., 1]

        def rot(x):                                    # [..., 64] fp32
            a, b = x[..., :half], x[..., half:]
            cc, ss = (c, s) if x.dim() == 2 else (c[:, None, :], s[:, None, :])
            return torch.cat([a * cc - b * ss, b * cc + a * ss], dim=-1)

        kf = kva.float()
        ck = kf[:, :dl]
        ck = ck * torch.rsqrt(ck.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()
        kr = rot(kf[:, dl:dl + dr])
        row = torch.cat([ck, kr], dim=-1).to(cache.dtype)
        ok = slots >= 0
        if bool(ok.any()):
            cache[slots[ok].long()] = row[ok]
        q[:, :, dl:] = rot(q[:, :, dl:].float()).to(q.dtype)
        return
    assert q.is_contiguous() and cache.is_contiguous() and kva.stride(1) == 1
    rc = _native.kernels().ib_mla_rope_kvwrite(q.data_ptr(), T, hq, kva.data_ptr(), kva.stride(0), pos.data_ptr(),
                                               slots.data_ptr(), cos_sin.data_ptr(), norm_w.data_ptr(), eps,
                                               cache.data_ptr(), K._stream())
    _native.check(rc, "ib_mla_rope_kvwrite")
    K._count(1)


def mla_attention(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, q_row: torch.Tensor,
                  q_kvlen: torch.Tensor, scale: float, splits: int | None = None, max_kvlen: int | None = None,
                  out: torch.Tensor | None = None, rope_dim: int = DR) -> torch.Tensor:
    """o [nq, hq, 512] = softmax(q . K^T * scale) V over each query's first
    ``q_kvlen`` cached keys (its block-table row ``q_row``); V = the first
    (width - rope_dim) dims of each cached row."""
    nq, hq, _ = q.shape
    if not q.is_cuda:
        dl = cache.shape[1] - rope_dim
        o = torch.zeros(nq, hq, dl, dtype=torch.float32)
        rows = q_row.tolist()
        lens = q_kvlen.tolist()
        for i in range(nq):
            L = int(lens[i])
            if L <= 0:
                continue
            pages = block_table[rows[i], : -(-L // PAGE)].long()
            slots = (pages[:, None] * PAGE + torch.arange(PAGE)).reshape(-1)[:L]
            kv = cache[slots].float()
            s = q[i].float() @ kv.t() * scale
            o[i] = torch.softmax(s, dim=-1) @ kv[:, :dl]
        o = o.to(torch.bfloat16)
        if out is not None:
            out.copy_(o)
            return out
        return o
    assert q.is_contiguous() and cache.is_contiguous() and cache.shape[1] == DQK and rope_dim == DR
    if out is None:
        out = torch.empty(nq, hq, DL, dtype=torch.bfloat16, device=q.device)
    if splits is None:
        splits = mla_splits(nq, max_kvlen if max_kvlen is not None else 8192, K._num_sms())
    o_part = lse = None
    if splits > 1:
        o_part = torch.empty(nq * splits * hq * DL, dtype=torch.float32, device=q.device)
        lse = torch.empty(nq * splits * hq, dtype=torch.float32, device=q.device)
    sc = K.scratch(q.device)
    rc = _native.kernels().ib_mla_decode(q.data_ptr(), nq, hq, cache.data_ptr(), cache.shape[0], q_row.data_ptr(),
                                         q_kvlen.data_ptr(), block_table.data_ptr(), block_table.shape[1], splits,
                                         scale, out.data_ptr(), K._ptr(o_part), K._ptr(lse), sc.status.data_ptr(),
                                         K._stream())
    _native.check(rc, "ib_mla_decode")
    K._count(2 if splits > 1 else 1)
    return out


def kv_up_weight(w_uk: torch.Tensor, w_uv: torch.Tensor) -> torch.Tensor:
    """[Hq * (dn + dv), L]: per head the rows of W_UK^T (k_nope = W_UK^T c)
    then W_UV (v = W_UV c), so one GEMM of the latent rows gives every
    head's [k_nope | v] side by side."""
    hq, L, dn = w_uk.shape
    return torch.cat([w_uk.transpose(1, 2), w_uv], dim=1).reshape(-1, L).contiguous()


def _compact_pages(block_table: torch.Tensor, bt_rows: torch.Tensor | None, ctx_lens: list[int],
                   device: torch.device) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Cache slots of every sequence's context pages, laid end to end, and a
    block table over that compact layout (row i = its pages' new ids)."""
    n_pages = [-(-c // PAGE) for c in ctx_lens]
    P = sum(n_pages)
    starts = [0]
    for n in n_pages[:-1]:
        starts.append(starts[-1] + n)
    n_seqs = len(ctx_lens)
    rows = bt_rows.long() if bt_rows is not None else torch.arange(n_seqs, device=device)
    cnt = torch.tensor(n_pages, device=device)
    start_t = torch.tensor(starts, device=device)
    seq_of = torch.repeat_interleave(torch.arange(n_seqs, device=device), cnt, output_size=P)
    j = torch.arange(P, device=device) - start_t[seq_of]
    pages = block_table[rows[seq_of], j].long()
    slots = (pages[:, None] * PAGE + torch.arange(PAGE, device=device)).reshape(-1).to(torch.int32)
    max_pc = max(n_pages)
    jj = torch.arange(max_pc, device=device)
    bt_c = (start_t[:, None] + torch.minimum(jj[None, :], (cnt - 1)[:, None])).to(torch.int32).contiguous()
    return slots, bt_c, P


def mla_prefill(qb: torch.Tensor, q_rope: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor,
                bt_rows: torch.Tensor | None, host_meta: tuple[list[int], list[int]], q_start: torch.Tensor,
                q_len: torch.Tensor, ctx_len: torch.Tensor, tiles: torch.Tensor, w_kv_up: torch.Tensor, hq: int,
                dn: int, dv: int, scale: float, out: torch.Tensor | None = None, dr: int = DR) -> torch.Tensor:
    """Causal MLA attention of prompt chunks, not absorbed.

    qb [Tp, hq * (dn + dr)]: per head the nope query then the raw rope
    query (only the nope part is read); q_rope [Tp, hq, >= dr] view whose
    last dims are the rotated rope queries (``mla_rope_kvwrite`` output);
    cache [slots, L + dr] latent rows already written for these tokens;
    host_meta = (q_lens, ctx_lens). Returns [Tp, hq * dv]."""
    qls, ctxs = host_meta
    Tp = qb.shape[0]
    L = cache.shape[1] - dr
    slots, bt_c, P = _compact_pages(block_table, bt_rows, ctxs, qb.device)
    compact = K.gather_rows(cache, slots)                       # [P*16, L + dr]
    kv_up = K.linear(compact[:, :L], w_kv_up)                  # [P*16, hq * (dn + dv)]
    w = dn + dv
    if not qb.is_cuda:
        o = torch.zeros(Tp, hq, dv, dtype=torch.float32)
        kvf = kv_up.float().view(-1, hq, w)
        kpe = compact[:, L:].float()
        row = 0
        for i, (n, c) in enumerate(zip(qls, ctxs)):
            pages = bt_c[i, : -(-c // PAGE)].long()
            idx = (pages[:, None] * PAGE + torch.arange(PAGE)).reshape(-1)[:c]
            kn, vv, kp = kvf[idx, :, :dn], kvf[idx, :, dn:], kpe[idx]       # [c, hq, dn], [c, hq, dv], [c, dr]
            qn = qb[row:row + n].float().view(n, hq, -1)[:, :, :dn]
            qp = q_rope[row:row + n].float()[:, :, -dr:]
            sc = (torch.einsum("thd,shd->hts", qn, kn) + torch.einsum("thd,sd->hts", qp, kp)) * scale
            qpos = torch.arange(c - n, c)
            sc = sc.masked_fill(torch.arange(c)[None, None, :] > qpos[None, :, None], float("-inf"))
            o[row:row + n] = torch.einsum("hts,shv->thv", torch.softmax(sc, -1), vv)
            row += n
        y = o.reshape(Tp, hq * dv).to(torch.bfloat16)
        if out is not None:
            out[:Tp].copy_(y)
            return out
        return y
    assert dn == 128 and dv == 128 and dr == DR and q_rope.stride(-1) == 1
    if out is None:
        out = torch.empty(Tp, hq * dv, dtype=torch.bfloat16, device=qb.device)
    qe = q_rope[..., -DR:]
    sc_ = K.scratch(qb.device)
    splits = K.prefill_kv_splits(hq, tiles.shape[0], max(ctxs), K._num_sms())
    o_ptr = lse_ptr = None
    if splits > 1:
        o_p, lse_p = sc_.ensure_prefill(Tp * hq * splits * 128, Tp * hq * splits)
        o_ptr, lse_ptr = o_p.data_ptr(), lse_p.data_ptr()
    rc = _native.kernels().ib_attn_prefill_ext(
        qb.data_ptr(), Tp, qb.stride(0), qb.shape[1] // hq,
        qe.data_ptr(), qe.stride(0), qe.stride(1),
        kv_up.data_ptr(), kv_up.stride(0), w,
        compact[:, L:].data_ptr(), compact.stride(0), 0,
        kv_up[:, dn:].data_ptr(), kv_up.stride(0), w,
        P * PAGE, tiles.data_ptr(), tiles.shape[0], q_start.data_ptr(), q_len.data_ptr(), ctx_len.data_ptr(),
        bt_c.data_ptr(), None, bt_c.shape[1], hq, hq, scale, out.data_ptr(), out.stride(0),
        sc_.status.data_ptr(), splits, o_ptr, lse_ptr, K._stream())
    _native.check(rc, "ib_attn_prefill_ext")
    K._count(2 if splits > 1 else 1)
    return out


def default_scale(qk_nope_dim: int, qk_rope_dim: int) -> float:
    return 1.0 / math.sqrt(qk_nope_dim + qk_rope_dim)

"""Multi-head latent attention ops (DeepSeek-V3 MLA, absorbed form).

* :func:`mla_rope_kvwrite` - RMS-normalise the compressed KV, rotate the
  shared rope key and every head's rope query, write the 576-wide latent
  row of each token into its cache slot (``ib_mla_rope_kvwrite``);
* :func:`mla_attention` - multi-query attention of the absorbed queries
  [nq, hq, 576] over the paged latent cache, values = the first 512 dims of
  each cached row (``ib_mla_decode``, tcgen05); split over the keys when
  few queries are in flight, merged by log-sum-exp.

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


def mla_splits(nq: int, max_kvlen: int, num_sms: int = 148) -> int:
    """Key splits per query: enough CTAs (nq x 2 value halves x splits) to
    cover the SMs, each split keeping at least 4 tiles of 32 keys."""
    tiles = max(1, -(-max_kvlen // 32))
    want = max(1, -(-num_sms // (2 * max(nq, 1))))
    return max(1, min(want, tiles // 4 if tiles >= 8 else 1, 64))


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


def default_scale(qk_nope_dim: int, qk_rope_dim: int) -> float:
    return 1.0 / math.sqrt(qk_nope_dim + qk_rope_dim)

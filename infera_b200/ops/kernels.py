"""Tensor-level entry points for the sm_100a kernels.

Every function takes and returns torch tensors. On CUDA tensors it calls the
native kernel from ``libib200_kernels.so`` (there is no library fallback on a
GPU). On CPU tensors it runs the plain fp32 PyTorch restatement of the same
op, which is also the oracle the GPU tests compare against.

Per-device scratch (the split-K fp32 workspace, the decode split-KV
partials and the kernel status word) lives in :class:`DeviceScratch`; the
engine sizes it once at start-up so that CUDA-graph capture never allocates.
"""

from __future__ import annotations

import math
import os as _os
from dataclasses import dataclass, field

import torch

from infera_b200.ops import _native

# ---------------------------------------------------------------- scratch


@dataclass
class DeviceScratch:
    device: torch.device
    status: torch.Tensor
    gemm_ws: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    dec_o: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    dec_lse: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    pf_o: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    pf_lse: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    # per-tile k-block counters of the in-kernel split reduction (uint32,
    # zero between GEMMs; the GEMM that completes a tile resets its counter)
    gemm_ctr: torch.Tensor = field(default_factory=lambda: torch.empty(0))

    # Growth is refused while a CUDA graph is being captured (a captured
    # kernel must keep pointing at live memory); engines size the scratch
    # before they capture.
    def ensure_gemm(self, numel: int) -> torch.Tensor:
        if self.gemm_ws.numel() < numel:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"GEMM workspace too small ({self.gemm_ws.numel()} < {numel}) during capture")
            self.gemm_ws = torch.zeros(numel, dtype=torch.float32, device=self.device)
        return self.gemm_ws

    def ensure_decode(self, o_numel: int, lse_numel: int) -> tuple[torch.Tensor, torch.Tensor]:
        if self.dec_o.numel() < o_numel or self.dec_lse.numel() < lse_numel:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("decode scratch too small during capture")
            self.dec_o = torch.empty(max(o_numel, self.dec_o.numel()), dtype=torch.float32, device=self.device)
            self.dec_lse = torch.empty(max(lse_numel, self.dec_lse.numel()), dtype=torch.float32,
                                       device=self.device)
        return self.dec_o, self.dec_lse

    def ensure_prefill(self, o_numel: int, lse_numel: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Partials of key-split prefill attention (prefill runs eagerly, never
        inside a captured graph, so this may grow at any time)."""
        if self.pf_o.numel() < o_numel or self.pf_lse.numel() < lse_numel:
            self.pf_o = torch.empty(max(o_numel, self.pf_o.numel()), dtype=torch.float32, device=self.device)
            self.pf_lse = torch.empty(max(lse_numel, self.pf_lse.numel()), dtype=torch.float32, device=self.device)
        return self.pf_o, self.pf_lse

    def read_status(self) -> int:
        return int(self.status[0].item())

    def read_status_detail(self) -> dict:
        """The first error's details (index checks): what (1 position, 2 KV
        slot, 3 token id), the token row, the offending value."""
        code, what, where, value = (int(v) for v in self.status.tolist())
        return {"code": code, "what": what, "where": where, "value": value}

    def clear_status(self) -> None:
        self.status.zero_()


_scratch: dict[int, DeviceScratch] = {}


def _probe_status() -> dict | None:
    idx = torch.cuda.current_device()
    s = _scratch.get(idx)
    return s.read_status_detail() if s is not None else None


_native.status_probe = _probe_status


def scratch(device: torch.device | int | None = None) -> DeviceScratch:
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx != torch.cuda.current_device():
        # launches go to the current device's stream: refuse instead of
        # faulting on another device's pointers
        raise RuntimeError(f"tensors on cuda:{idx} but this thread's current device is "
                           f"cuda:{torch.cuda.current_device()} (call torch.cuda.set_device first)")
    s = _scratch.get(idx)
    if s is None:
        dev = torch.device("cuda", idx)
        # the status word, then three ints of details of the first error
        s = DeviceScratch(device=dev, status=torch.zeros(4, dtype=torch.int32, device=dev))
        if _FUSED_REDUCE:
            s.gemm_ctr = torch.zeros(_GEMM_CTRS, dtype=torch.int32, device=dev)
            _native.kernels().ib_gemm_set_tile_counters(s.gemm_ctr.data_ptr(), _GEMM_CTRS)
        _scratch[idx] = s
    return s


# Number of kernel launches issued through this module (graph replays add
# the launches captured in the graph); used to report launch counts.
LAUNCHES = [0]
_plan_cache: dict[tuple[int, int, int, int], int] = {}


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def _gemm_plan_splits(M: int, N: int, K: int, force_split: int = 0) -> int:
    """The plan's split-K factor, or -1 for a stream-K plan."""
    key = (M, N, K, force_split)
    v = _plan_cache.get(key)
    if v is None:
        v = gemm_plan(M, N, K, _num_sms(), force_split)["splits"]
        _plan_cache[key] = v
    return v


def _gemm_splits(M: int, N: int, K: int, force_split: int = 0) -> int:
    """K splits of the plan (1 for stream-K, whose shares are uneven)."""
    return max(1, _gemm_plan_splits(M, N, K, force_split))


def _gemm_ws(M: int, N: int, K: int, force_split: int = 0) -> bool:
    """Whether the plain GEMM accumulates in the fp32 workspace (split-K or
    stream-K) and runs the finalize pass."""
    v = _gemm_plan_splits(M, N, K, force_split)
    return v > 1 or v < 0


# INFERA_GEMM_FUSED_REDUCE=1: split-K / stream-K partial sums are reduced
# inside the GEMM (the CTA that completes a tile reads it back and stores
# it) instead of by the finalize kernel. Off by default: on B200 the
# read-back sits on the completing CTA's critical path and measured slower
# (64 x 28672 x 4096 stream-K 0.072 vs 0.056 ms; 288 x 4096 x 14336 split-K
# 0.371 vs 0.052 ms).
_FUSED_REDUCE = _os.environ.get("INFERA_GEMM_FUSED_REDUCE", "0") == "1"
_GEMM_CTRS = 1 << 16


def _gemm_launches(M: int, N: int, K: int, force_split: int = 0) -> int:
    return 1 + (1 if _gemm_ws(M, N, K, force_split) and not _FUSED_REDUCE else 0)


_NUM_SMS: list[int] = []


def _num_sms() -> int:
    if not _NUM_SMS:
        _NUM_SMS.append(torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
                        if torch.cuda.is_available() else 148)
    return _NUM_SMS[0]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------- GEMM


def gemm_plan(M: int, N: int, K: int, num_sms: int = 148, force_split: int = 0) -> dict:
    out = (_native.c_int * 7)()
    _native.kernels().ib_gemm_bf16_plan(M, N, K, num_sms, force_split, out)
    keys = ["swap", "bn", "p_tiles", "q_tiles", "splits", "kbps", "grid"]
    return dict(zip(keys, list(out)))


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, swiglu: bool = False,
           force_split: int = 0) -> torch.Tensor:
    """y = x @ w.T (bf16 in/out, fp32 accumulate).

    ``swiglu=True`` expects ``w`` rows interleaved as (gate_0, up_0, gate_1,
    up_1, ...) and returns silu(gate) * up with half the columns.
    """
    if not isinstance(w, torch.Tensor):  # fp8 block-scaled weight
        from infera_b200.ops import fp8

        return fp8.linear(x, w, out=out, swiglu=swiglu)
    M, K = x.shape
    N = w.shape[0]
    n_out = N // 2 if swiglu else N
    if not x.is_cuda:
        y = x.float() @ w.float().t()
        if swiglu:
            g, u = y[:, 0::2], y[:, 1::2]
            y = torch.nn.functional.silu(g) * u
        y = y.to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    assert x.stride(1) == 1 and w.stride(1) == 1
    if out is None:
        out = torch.empty(M, n_out, dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return out
    sc = scratch(x.device)
    ws = sc.ensure_gemm(M * N if _gemm_ws(M, N, K, force_split) else 1)
    rc = _native.kernels().ib_gemm_bf16(x.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, K, x.stride(0),
                                        w.stride(0), out.stride(0), 1 if swiglu else 0, ws.data_ptr(),
                                        force_split, sc.status.data_ptr(), _stream())
    _native.check(rc, "ib_gemm_bf16")
    _count(_gemm_launches(M, N, K, force_split))
    return out


# A split GEMM's consumer can read its fp32 workspace itself (and zero it)
# instead of a finalize launch (INFERA_GEMM_DEFER=0: always finalize). A
# graphed Llama-3.1-8B decode step of 48 sequences: 7.22 ms against 7.44 ms.
_DEFER = _os.environ.get("INFERA_GEMM_DEFER", "1") != "0"


def linear_deferred(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor | None:
    """y = x @ w.T for a consumer that can take the fp32 workspace: returns
    the workspace view [M, N] (fp32, not rounded, the consumer zeroes it)
    when the GEMM was split, else None with y in ``out`` (bf16)."""
    M, Kd = x.shape
    N = w.shape[0]
    if not x.is_cuda or not _DEFER or not isinstance(w, torch.Tensor) or M == 0 or not _gemm_ws(M, N, Kd):
        linear(x, w, out=out)
        return None
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    assert x.stride(1) == 1 and w.stride(1) == 1
    sc = scratch(x.device)
    ws = sc.ensure_gemm(M * N)
    in_ws = (_native.c_int * 1)()
    rc = _native.kernels().ib_gemm_bf16_deferred(x.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, Kd, x.stride(0),
                                                 w.stride(0), out.stride(0), ws.data_ptr(), sc.status.data_ptr(),
                                                 in_ws, _stream())
    _native.check(rc, "ib_gemm_bf16_deferred")
    _count(1)
    return ws[: M * N].view(M, N) if in_ws[0] else None


def add_rmsnorm_ws(ws: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                   out: torch.Tensor) -> torch.Tensor:
    """residual += bf16(ws) (ws: a split GEMM's fp32 [T, H] workspace view,
    zeroed here); return rmsnorm(residual) * w."""
    T, H = residual.shape
    rc = _native.kernels().ib_add_rmsnorm_ws(ws.data_ptr(), ws.stride(0), residual.data_ptr(), w.data_ptr(),
                                             out.data_ptr(), T, H, residual.stride(0), out.stride(0), eps, _stream())
    _native.check(rc, "ib_add_rmsnorm_ws")
    _count()
    return out


def rope_kvwrite_ws(ws: torch.Tensor, qkv: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor,
                    cos_sin: torch.Tensor, hq: int, hkv: int, head_dim: int, k_cache: torch.Tensor,
                    v_cache: torch.Tensor) -> None:
    """rope_kvwrite over a split GEMM's fp32 qkv workspace view [T, N]
    (zeroed here): rotated q heads into ``qkv``, k and v into the caches."""
    T = qkv.shape[0]
    rc = _native.kernels().ib_rope_kvwrite_ws(ws.data_ptr(), ws.stride(0), qkv.data_ptr(), T, qkv.stride(0),
                                              pos.data_ptr(), slots.data_ptr(), cos_sin.data_ptr(), hq, hkv,
                                              head_dim, k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0),
                                              k_cache.shape[0], cos_sin.shape[0],
                                              scratch(qkv.device).status.data_ptr(), _stream())
    _native.check(rc, "ib_rope_kvwrite_ws")
    _count()


# ---------------------------------------------------------------- norms / rope / embed


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    if not x.is_cuda:
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
        y = y.to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, H = x.shape
    if out is None:
        out = torch.empty_like(x)
    rc = _native.kernels().ib_rmsnorm(x.data_ptr(), w.data_ptr(), out.data_ptr(), T, H, x.stride(0), out.stride(0),
                                      eps, _stream())
    _native.check(rc, "ib_rmsnorm")
    _count()
    return out


def add_rmsnorm(delta: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """residual += delta (in place, bf16); return rmsnorm(residual) * w."""
    if not residual.is_cuda:
        residual.copy_((residual.float() + delta.float()).to(residual.dtype))
        return rmsnorm(residual, w, eps, out)
    T, H = residual.shape
    if out is None:
        out = torch.empty_like(residual)
    rc = _native.kernels().ib_add_rmsnorm(delta.data_ptr(), residual.data_ptr(), w.data_ptr(), out.data_ptr(), T, H,
                                          delta.stride(0), residual.stride(0), out.stride(0), eps, _stream())
    _native.check(rc, "ib_add_rmsnorm")
    _count()
    return out


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, scaling: dict | None = None,
                 device: torch.device | str = "cpu") -> torch.Tensor:
    """[max_pos, head_dim/2, 2] fp32 (cos, sin) table, with optional
    Llama-3 frequency scaling (factor, low/high_freq_factor,
    original_max_position_embeddings)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling:
        factor = scaling.get("factor", 8.0)
        lo = scaling.get("low_freq_factor", 1.0)
        hi = scaling.get("high_freq_factor", 4.0)
        orig = scaling.get("original_max_position_embeddings", 8192)
        lo_wl, hi_wl = orig / lo, orig / hi
        wl = 2 * math.pi / inv
        smooth = (orig / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        scaled = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        inv = scaled
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    cs = torch.stack([f.cos(), f.sin()], dim=-1).to(torch.float32)
    return cs.to(device)


def rope_kvwrite(qkv: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor, cos_sin: torch.Tensor, hq: int,
                 hkv: int, head_dim: int, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    """Rotate q/k of ``qkv`` in place and store k, v at ``slots`` of the
    caches ([num_slots, hkv*head_dim]); slot -1 skips the store."""
    T = qkv.shape[0]
    if not qkv.is_cuda:
        half = head_dim // 2
        cs = cos_sin[pos.long()]  # [T, half, 2]
        c, s = cs[..., 0], cs[..., 1]
        x = qkv[:, : (hq + hkv) * head_dim].float().view(T, hq + hkv, head_dim)
        a, b = x[..., :half], x[..., half:]
        c, s = c[:, None, :], s[:, None, :]
        ra, rb = a * c - b * s, b * c + a * s
        rot = torch.cat([ra, rb], dim=-1).to(qkv.dtype).view(T, -1)
        qkv[:, : (hq + hkv) * head_dim] = rot
        keep = slots >= 0
        if keep.any():
            idx = slots[keep].long()
            k = qkv[keep, hq * head_dim:(hq + hkv) * head_dim]
            v = qkv[keep, (hq + hkv) * head_dim:(hq + 2 * hkv) * head_dim]
            k_cache[idx] = k
            v_cache[idx] = v
        return
    rc = _native.kernels().ib_rope_kvwrite(qkv.data_ptr(), T, qkv.stride(0), pos.data_ptr(), slots.data_ptr(),
                                           cos_sin.data_ptr(), hq, hkv, head_dim, k_cache.data_ptr(),
                                           v_cache.data_ptr(), k_cache.stride(0), k_cache.shape[0], cos_sin.shape[0],
                                           scratch(qkv.device).status.data_ptr(), _stream())
    _native.check(rc, "ib_rope_kvwrite")
    _count()


def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if not table.is_cuda:
        y = table[ids.long()]
        if out is not None:
            out.copy_(y)
            return out
        return y
    T = ids.shape[0]
    H = table.shape[1]
    if out is None:
        out = torch.empty(T, H, dtype=table.dtype, device=table.device)
    rc = _native.kernels().ib_embed(ids.data_ptr(), table.data_ptr(), out.data_ptr(), T, H, table.shape[0],
                                    scratch(ids.device).status.data_ptr(), _stream())
    _native.check(rc, "ib_embed")
    _count()
    return out


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if not src.is_cuda:
        y = src[idx.long()]
        if out is not None:
            out.copy_(y)
            return out
        return y
    n = idx.shape[0]
    if out is None:
        out = torch.empty(n, src.shape[1], dtype=src.dtype, device=src.device)
    rc = _native.kernels().ib_gather_rows(src.data_ptr(), idx.data_ptr(), out.data_ptr(), n, src.stride(0),
                                          _stream())
    _native.check(rc, "ib_gather_rows")
    _count()
    return out


def _mix64(z: torch.Tensor) -> torch.Tensor:
    # same splitmix64 finaliser as the kernel, on uint64 emulated in int64
    m = (1 << 64) - 1
    z = [int(v) & m for v in z.tolist()]
    out = []
    for v in z:
        v = (v + 0x9E3779B97F4A7C15) & m
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m
        out.append(v ^ (v >> 31))
    return out


def sample(logits: torch.Tensor, temperature: torch.Tensor | None = None, seeds: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy (temperature 0) or Gumbel-max sampling per row -> int32 ids."""
    B, V = logits.shape
    if not logits.is_cuda:
        x = logits.float()
        if temperature is not None and bool((temperature > 0).any()):
            res = []
            for b in range(B):
                T = float(temperature[b])
                if T <= 0:
                    res.append(int(torch.argmax(x[b])))
                    continue
                seed = int(seeds[b]) if seeds is not None else 0
                m = (1 << 64) - 1
                keys = [((seed * 0x100000001B3) & m) ^ i for i in range(V)]
                hs = _mix64(torch.tensor([k if k < (1 << 63) else k - (1 << 64) for k in keys]))
                u = torch.tensor([((h >> 40) + 0.5) / 16777216.0 for h in hs], dtype=torch.float32)
                g = x[b] / T - torch.log(-torch.log(u))
                res.append(int(torch.argmax(g)))
            y = torch.tensor(res, dtype=torch.int32)
        else:
            y = torch.argmax(x, dim=-1).to(torch.int32)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    rc = _native.kernels().ib_sample(logits.data_ptr(), B, logits.stride(0), V, _ptr(temperature), _ptr(seeds),
                                     out.data_ptr(), _stream())
    _native.check(rc, "ib_sample")
    _count()
    return out


# ---------------------------------------------------------------- attention


def _ref_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                   q_pos: list[list[int]], ctx_lens: list[int], hq: int, hkv: int, scale: float,
                   page: int = 16) -> list[torch.Tensor]:
    """fp32 oracle: for each sequence, q rows [n_i, hq*D] attend causally to
    the first ctx_len keys of its pages. Returns a list of [n_i, hq*D]."""
    D = k_cache.shape[1] // hkv
    G = hq // hkv
    outs = []
    row = 0
    for i, ctx in enumerate(ctx_lens):
        n = len(q_pos[i])
        pages = block_table[i, : (ctx + page - 1) // page].long()
        slots = (pages[:, None] * page + torch.arange(page)[None, :]).reshape(-1)[:ctx]
        k = k_cache[slots].float().view(ctx, hkv, D)
        v = v_cache[slots].float().view(ctx, hkv, D)
        qi = q[row: row + n].float().view(n, hq, D)
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        s = torch.einsum("nhd,khd->hnk", qi, k) * scale
        pos = torch.tensor(q_pos[i])[:, None]
        mask = torch.arange(ctx)[None, :] > pos
        s = s.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("hnk,khd->nhd", p, v).reshape(n, hq * D)
        outs.append(o)
        row += n
    return outs


# Decode attention splits every sequence into chunks of this many 128-key
# tiles at the same absolute positions (INFERA_DECODE_TPS=0: divide each
# sequence evenly over decode_splits() splits instead).

DECODE_TILES_PER_SPLIT = int(_os.environ.get("INFERA_DECODE_TPS", "16"))


def decode_plan(batch: int, hkv: int, max_len: int) -> tuple[int, int]:
    """(splits, tiles per split) of the decode attention for a batch whose
    longest sequence has ``max_len`` keys."""
    tps = DECODE_TILES_PER_SPLIT
    if tps <= 0:
        return decode_splits(batch, hkv, max_len), 0
    tiles = max(1, (max_len + 127) // 128)
    return max(1, -(-tiles // tps)), tps


def decode_splits(batch: int, hkv: int, max_len: int, num_sms: int = 148) -> int:
    """Split-KV factor: enough CTAs for ~2 waves, at least 4 tiles per split."""
    ctas = max(1, batch * hkv)
    want = max(1, (2 * num_sms + ctas - 1) // ctas)
    tiles = max(1, (max_len + 63) // 64)
    return int(max(1, min(want, (tiles + 3) // 4, 64)))


def attn_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                seq_lens: torch.Tensor, hq: int, hkv: int, scale: float, splits: int = 1,
                out: torch.Tensor | None = None, bt_rows: torch.Tensor | None = None,
                impl: str = "tc", tiles_per_split: int = 0, l2_policy: int = 0) -> torch.Tensor:
    """Single-token attention per sequence. q: [B, >=hq*D] (row stride
    free), seq_lens: int32 [B] (keys including the current token).

    ``impl="tc"`` is the tcgen05/TMA kernel the engine uses; ``"simt"`` is
    the FP32-pipe kernel behind the allocation-free C entry point.
    ``tiles_per_split`` > 0: split s covers 128-key tiles [s*T, (s+1)*T) of
    every sequence (``splits * T * 128`` must cover the longest), so CTAs
    reading a shared prefix run together; ``l2_policy`` 0/1/2: K/V loads
    evict_first / evict_normal / evict_last."""
    B = seq_lens.shape[0]
    D = k_cache.shape[1] // hkv
    if not q.is_cuda:
        lens = [int(x) for x in seq_lens.tolist()]
        bt = block_table if bt_rows is None else block_table[bt_rows.long()]
        outs = _ref_attention(q[:, : hq * D], k_cache, v_cache, bt, [[n - 1] for n in lens], lens, hq, hkv, scale)
        y = torch.cat(outs, 0).to(q.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(B, hq * D, dtype=q.dtype, device=q.device)
    o_ptr = lse_ptr = None
    sc = scratch(q.device)
    if splits > 1:
        o, lse = sc.ensure_decode(B * hq * splits * D, B * hq * splits)
        o_ptr, lse_ptr = o.data_ptr(), lse.data_ptr()
    if impl == "tc":
        rc = _native.kernels().ib_attn_decode_tc_ex(q.data_ptr(), q.stride(0), k_cache.data_ptr(),
                                                    v_cache.data_ptr(), k_cache.shape[0], block_table.data_ptr(),
                                                    _ptr(bt_rows), seq_lens.data_ptr(), block_table.stride(0), B, hq,
                                                    hkv, splits, scale, o_ptr, lse_ptr, out.data_ptr(), out.stride(0),
                                                    sc.status.data_ptr(), tiles_per_split, l2_policy, _stream())
        _native.check(rc, "ib_attn_decode_tc")
    else:
        rc = _native.kernels().ib_attn_decode(q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                              block_table.data_ptr(), _ptr(bt_rows), seq_lens.data_ptr(),
                                              block_table.stride(0), B, hq, hkv, splits, scale, o_ptr, lse_ptr,
                                              out.data_ptr(), out.stride(0), _stream())
        _native.check(rc, "ib_attn_decode")
    _count(2 if splits > 1 else 1)
    return out


# Query rows per prefill attention CTA: 256 runs two 128-row tiles per CTA
# that share every K / V tile and alternate on the tensor core (128-dim
# heads); 128 runs one tile (INFERA_PREFILL_TILE_ROWS=128).
PREFILL_TILE_ROWS = int(_os.environ.get("INFERA_PREFILL_TILE_ROWS", "256"))


def prefill_tiles(q_lens: list[int], rows: int | None = None) -> list[tuple[int, int]]:
    """(seq, q_block) work items of ``rows`` query rows (q_block counts
    128-row blocks; a 256-row item covers q_block and q_block + 1),
    longest-work first."""
    step = (rows or PREFILL_TILE_ROWS) // 128
    items = []
    for s, n in enumerate(q_lens):
        for b in range(0, (n + 127) // 128, step):
            items.append((s, b))
    # later blocks of long sequences see more keys; schedule them first
    items.sort(key=lambda it: -(it[1]))
    return items


def prefill_kv_splits(num_heads: int, num_tiles: int, max_ctx: int, num_sms: int = 148) -> int:
    """Key shares per (head, query tile) CTA, when the CTAs do not fill one
    wave of SMs (a short chunk over a long cached context): the share count
    that minimises the work on the busiest SM, waves x (key tiles per share
    + two tiles' worth of start-up and combine), fewest shares on a tie, at
    least 4 key tiles of 128 per share. (A 1024-query chunk over 8192 keys,
    128 two-tile CTAs, runs 0.157 ms unsplit against 0.204 ms in 3 shares.)"""
    ctas = num_heads * num_tiles
    kv_tiles = -(-max_ctx // 128)
    if ctas >= num_sms or kv_tiles < 16:
        return 1
    best, best_cost = 1, None
    for sp in range(1, min(16, kv_tiles // 4) + 1):
        cost = -(-ctas * sp // num_sms) * (-(-kv_tiles // sp) + 2)
        if best_cost is None or cost < best_cost:
            best, best_cost = sp, cost
    return best


def attn_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                 q_start: torch.Tensor, q_len: torch.Tensor, ctx_len: torch.Tensor, tiles: torch.Tensor, hq: int,
                 hkv: int, scale: float, out: torch.Tensor | None = None,
                 host_meta: tuple[list[int], list[int]] | None = None,
                 bt_rows: torch.Tensor | None = None, kv_splits: int | None = None,
                 tile_rows: int | None = None) -> torch.Tensor:
    """Causal attention for chunks of new tokens whose K/V already sit in the
    paged cache. q: [T, >=hq*D]; q_start/q_len/ctx_len: int32 [num_seqs];
    tiles: int32 [num_tiles, 2] from :func:`prefill_tiles` with the same
    ``tile_rows`` (None: ``PREFILL_TILE_ROWS``). ``kv_splits``: key shares
    per tile (None: :func:`prefill_kv_splits` from ``host_meta``, 1 without
    it)."""
    T = q.shape[0]
    D = k_cache.shape[1] // hkv
    if not q.is_cuda:
        if host_meta is None:
            host_meta = ([int(x) for x in q_len.tolist()], [int(x) for x in ctx_len.tolist()])
        qls, ctxs = host_meta
        q_pos = [list(range(c - n, c)) for n, c in zip(qls, ctxs)]
        bt = block_table if bt_rows is None else block_table[bt_rows.long()]
        outs = _ref_attention(q[:, : hq * D], k_cache, v_cache, bt, q_pos, ctxs, hq, hkv, scale)
        y = torch.cat(outs, 0).to(q.dtype)
        if out is not None:
            out[: y.shape[0]].copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(T, hq * D, dtype=q.dtype, device=q.device)
    sc = scratch(q.device)
    if kv_splits is None:
        kv_splits = prefill_kv_splits(hq, tiles.shape[0], max(host_meta[1]), _num_sms()) if host_meta else 1
    o_ptr = lse_ptr = None
    if kv_splits > 1:
        o, lse = sc.ensure_prefill(T * hq * kv_splits * D, T * hq * kv_splits)
        o_ptr, lse_ptr = o.data_ptr(), lse.data_ptr()
    rc = _native.kernels().ib_attn_prefill(q.data_ptr(), T, q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                           k_cache.shape[0], tiles.data_ptr(), tiles.shape[0], q_start.data_ptr(),
                                           q_len.data_ptr(), ctx_len.data_ptr(), block_table.data_ptr(),
                                           _ptr(bt_rows), block_table.stride(0), hq, hkv, scale, out.data_ptr(),
                                           out.stride(0), sc.status.data_ptr(), kv_splits, o_ptr, lse_ptr,
                                           tile_rows or PREFILL_TILE_ROWS, _stream())
    _native.check(rc, "ib_attn_prefill")
    _count(2 if kv_splits > 1 else 1)
    return out


def scatter_i32(dst: torch.Tensor, idx: torch.Tensor, val: torch.Tensor) -> None:
    """dst.view(-1)[idx] = val (int32)."""
    n = idx.shape[0]
    if n == 0:
        return
    if not dst.is_cuda:
        dst.view(-1)[idx.long()] = val
        return
    rc = _native.kernels().ib_scatter_i32(dst.data_ptr(), idx.data_ptr(), val.data_ptr(), n, _stream())
    _native.check(rc, "ib_scatter_i32")
    _count()


def kv_channels(k_cache: torch.Tensor, v_cache: torch.Tensor) -> int:
    """2 for a K/V cache pair, 1 for a latent (MLA) cache, whose V tensor is
    a placeholder (one row per token holds the compressed KV and rope key)."""
    return 2 if v_cache.shape == k_cache.shape else 1


def kv_page_copy(k_cache: torch.Tensor, v_cache: torch.Tensor, chunk: torch.Tensor, pages: torch.Tensor,
                 page_size: int = 16, gather: bool = True, page_major: bool = False) -> None:
    """Move whole KV pages between the cache ([L, slots, H] per channel) and a
    contiguous chunk [C, L, n_pages*page_size, H] (C = :func:`kv_channels`),
    or with ``page_major`` [n_pages, C, L, page_size, H] (one chunk payload
    per page): ``gather=True`` copies cache -> chunk (save), ``False`` chunk
    -> cache (load)."""
    n = pages.shape[0]
    if n == 0:
        return
    L, slots, H = k_cache.shape
    C = kv_channels(k_cache, v_cache)
    if not k_cache.is_cuda:
        idx = (pages.long()[:, None] * page_size + torch.arange(page_size)[None, :]).reshape(-1)
        for c, cache in enumerate((k_cache, v_cache)[:C]):
            if page_major:
                view = chunk.view(n, C, L, page_size, H)
                if gather:
                    view[:, c] = cache[:, idx].view(L, n, page_size, H).permute(1, 0, 2, 3)
                else:
                    cache[:, idx] = view[:, c].permute(1, 0, 2, 3).reshape(L, n * page_size, H)
            else:
                view = chunk.view(C, L, n * page_size, H)
                if gather:
                    view[c] = cache[:, idx]
                else:
                    cache[:, idx] = view[c]
        return
    assert page_size == 16 and chunk.is_contiguous()
    rc = _native.kernels().ib_kv_page_copy(k_cache.data_ptr(), v_cache.data_ptr(), chunk.data_ptr(),
                                           pages.data_ptr(), n, L, slots, H, k_cache.element_size(), C,
                                           (0 if gather else 1) | (2 if page_major else 0), _stream())
    _native.check(rc, "ib_kv_page_copy")
    _count()


def kv_push_pages(src_k: torch.Tensor, src_v: torch.Tensor, dst_k, dst_v, src_pages: torch.Tensor,
                  dst_pages: torch.Tensor, layers: tuple[int, int] | None = None, dst_slots: int | None = None,
                  page_size: int = 16) -> None:
    """Copy whole KV pages of layers [l0, l1) from ``src_*`` ([L, slots, H]
    tensors) into ``dst_*``: tensors on this device, or raw device pointers
    (ints, CUDA-IPC mappings of another instance's caches; then
    ``dst_slots`` is required). A latent cache (one channel) pushes
    ``src_k`` only; ``dst_v`` may then be anything."""
    n = src_pages.shape[0]
    if n == 0:
        return
    L, slots, H = src_k.shape
    C = kv_channels(src_k, src_v)
    l0, l1 = layers if layers is not None else (0, L)
    if not src_k.is_cuda:
        idx_s = (src_pages.long()[:, None] * page_size + torch.arange(page_size)[None, :]).reshape(-1)
        idx_d = (dst_pages.long()[:, None] * page_size + torch.arange(page_size)[None, :]).reshape(-1)
        for s, d in ((src_k, dst_k), (src_v, dst_v))[:C]:
            d[l0:l1, idx_d] = s[l0:l1, idx_s]
        return
    assert page_size == 16
    if isinstance(dst_k, torch.Tensor):
        dst_slots = dst_k.shape[1]
        dk, dv = dst_k.data_ptr(), dst_v.data_ptr()
    else:
        assert dst_slots is not None
        dk, dv = int(dst_k), int(dst_v or 0)
    rc = _native.kernels().ib_kv_push_pages(src_k.data_ptr(), src_v.data_ptr(), dk, dv, src_pages.data_ptr(),
                                            dst_pages.data_ptr(), n, l0, l1, slots, dst_slots, H,
                                            src_k.element_size(), C, _stream())
    _native.check(rc, "ib_kv_push_pages")
    _count()


# ---------------------------------------------------------------- mixture of experts


def moe_topk(logits: torch.Tensor, top_k: int, n_groups: int = 1, topk_groups: int = 1,
             bias: torch.Tensor | None = None, scaling: float = 1.0, renorm: bool = True,
             softmax: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Router logits [T, E] -> (expert ids int32 [T, k], weights fp32 [T, k]):
    sigmoid (or softmax) scores, grouped selection on score + bias (groups
    ranked by their two best), weights = chosen scores, renormalised, x scaling."""
    T, E = logits.shape
    if not logits.is_cuda:
        x = logits.float()
        s = torch.softmax(x, -1) if softmax else torch.sigmoid(x)
        c = s + (bias.float() if bias is not None else 0.0)
        gs = E // n_groups
        if n_groups > 1:
            grp = c.view(T, n_groups, gs).topk(min(2, gs), dim=-1).values.sum(-1)
            keep = torch.zeros(T, n_groups, dtype=torch.bool)
            keep.scatter_(1, grp.topk(topk_groups, dim=-1).indices, True)
            c = c.masked_fill(~keep.repeat_interleave(gs, dim=1), float("-inf"))
        ids = c.topk(top_k, dim=-1).indices
        w = s.gather(1, ids)
        if renorm:
            w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
        return ids.to(torch.int32), (w * scaling).float()
    ids = torch.empty(T, top_k, dtype=torch.int32, device=logits.device)
    wts = torch.empty(T, top_k, dtype=torch.float32, device=logits.device)
    rc = _native.kernels().ib_moe_topk(logits.data_ptr(), logits.stride(0), 1 if logits.dtype == torch.bfloat16 else 0,
                                       _ptr(bias), T, E, n_groups, topk_groups, top_k, 1 if softmax else 0,
                                       1 if renorm else 0, scaling, ids.data_ptr(), wts.data_ptr(), _stream())
    _native.check(rc, "ib_moe_topk")
    _count()
    return ids, wts


def moe_permute(ids: torch.Tensor, E: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(offsets [E+1], row_of_slot [T*k], token_of_row [T*k]) int32: the
    expert-sorted row of every (token, slot) and each row's token."""
    T, k = ids.shape
    n = T * k
    dev = ids.device
    if not ids.is_cuda:
        flat = ids.reshape(-1).long()
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=E)
        offsets = torch.zeros(E + 1, dtype=torch.int32)
        offsets[1:] = torch.cumsum(counts, 0).to(torch.int32)
        row_of_slot = torch.empty(n, dtype=torch.int32)
        row_of_slot[order] = torch.arange(n, dtype=torch.int32)
        token_of_row = (order // k).to(torch.int32)
        return offsets, row_of_slot, token_of_row
    ws = torch.empty(2 * E + (E + 1) + 2 * n, dtype=torch.int32, device=dev)
    counts, cursor = ws[:E], ws[E:2 * E]
    offsets = ws[2 * E:3 * E + 1]
    row_of_slot = ws[3 * E + 1:3 * E + 1 + n]
    token_of_row = ws[3 * E + 1 + n:]
    rc = _native.kernels().ib_moe_permute(ids.data_ptr(), T, k, E, counts.data_ptr(), cursor.data_ptr(),
                                          offsets.data_ptr(), row_of_slot.data_ptr(), token_of_row.data_ptr(),
                                          _stream())
    _native.check(rc, "ib_moe_permute")
    _count(3)
    return offsets, row_of_slot, token_of_row


def grouped_bn(rows: int, E: int) -> int:
    avg = max(1, rows // max(1, E))
    for b in (16, 32, 64, 128):
        if avg <= b:
            return b
    return 256


def grouped_tiles(offsets: torch.Tensor, E: int, N: int, bn: int, R: int) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Device tile table of a grouped GEMM (``ib_moe_tiles``): (table, count, capacity)."""
    cap = (-(-R // bn) + E) * (N // 128)
    tab = torch.empty(cap * 4 + 1, dtype=torch.int32, device=offsets.device)
    num = tab[cap * 4:]
    _native.check(_native.kernels().ib_moe_tiles(offsets.data_ptr(), E, N, bn, tab.data_ptr(), num.data_ptr(),
                                                 _stream()), "ib_moe_tiles")
    _count(1)
    return tab, num, cap


def gemm_grouped(xp: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor, swiglu: bool = False,
                 out: torch.Tensor | None = None, bn: int | None = None) -> torch.Tensor:
    """Rows of ``xp`` [R, K] sorted by expert (``offsets`` [E+1]) times their
    expert's weight ``w`` [E, N, K]: out [R, N] (N/2 with ``swiglu``; gate
    and up rows interleaved per expert as in the dense layers)."""
    R, Kd = xp.shape
    E, N, _ = w.shape
    n_out = N // 2 if swiglu else N
    if not xp.is_cuda:
        y = torch.empty(R, N, dtype=torch.float32)
        off = offsets.tolist()
        for e in range(E):
            a, b = off[e], off[e + 1]
            if b > a:
                y[a:b] = xp[a:b].float() @ w[e].float().t()
        if swiglu:
            y = torch.nn.functional.silu(y[:, 0::2]) * y[:, 1::2]
        y = y.to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(R, n_out, dtype=torch.bfloat16, device=xp.device)
    bn = bn or grouped_bn(R, E)
    tab, num, cap = grouped_tiles(offsets, E, N, bn, R)
    lib = _native.kernels()
    sc = scratch(xp.device)
    rc = lib.ib_gemm_grouped(xp.data_ptr(), w.data_ptr(), out.data_ptr(), R, N, Kd, E, xp.stride(0), w.stride(1),
                             out.stride(0), 1 if swiglu else 0, tab.data_ptr(), num.data_ptr(), bn, cap,
                             sc.status.data_ptr(), _stream())
    _native.check(rc, "ib_gemm_grouped")
    _count(1)
    return out


def moe_combine(rows: torch.Tensor, row_of_slot: torch.Tensor, wts: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    T, k = wts.shape
    H = rows.shape[1]
    if not rows.is_cuda:
        g = rows.float()[row_of_slot.long()].view(T, k, H)
        y = (g * wts.float()[:, :, None]).sum(1).to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=rows.device)
    rc = _native.kernels().ib_moe_combine(rows.data_ptr(), rows.stride(0), row_of_slot.data_ptr(), wts.data_ptr(), T,
                                          k, H, out.data_ptr(), out.stride(0), _stream())
    _native.check(rc, "ib_moe_combine")
    _count()
    return out

"""W8A8 fp8 (e4m3) linear layers with power-of-two block scales.

Format (the DeepSeek-V3 / Llama-FP8 block-scaled layout with UE8M0 scales,
which Blackwell's block-scaled tensor-core MMA consumes directly):

* weights ``q`` [N, K] e4m3 and ``sf`` [ceil(N/128), K/128] uint8: one
  scale 2^(sf-127) per 128x128 block;
* activations ``q`` [M, K] e4m3 and ``sf`` [K/128, M] uint8: one scale per
  token and 128-wide K group, K-group-major (quantised on the fly by
  ``ib_quant_fp8_act``).

A scale is the smallest power of two that brings the block's largest
magnitude to at most 448 (e4m3's largest finite value); all-zero blocks
get scale 1. ``gemm_fp8`` runs ``ib_gemm_fp8`` (tcgen05
``kind::mxf8f6f4.block_scale``); on CPU every function computes the same
values with PyTorch (dequantise, fp32 matmul).

Reference counterpart: the 70B and DeepSeek-V3 configurations serve fp8
checkpoints with 128x128 block scales through their engines' fp8 GEMMs
(AITER / vLLM block-scaled W8A8); this module is that layer.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from infera_b200.ops import _native
from infera_b200.ops import kernels as K

E4M3_MAX = 448.0
GROUP = 128


@dataclass
class FP8Weight:
    q: torch.Tensor   # [N, K] float8_e4m3fn
    sf: torch.Tensor  # [ceil(N/128), K/128] uint8

    @property
    def shape(self) -> torch.Size:
        return self.q.shape

    @property
    def device(self) -> torch.device:
        return self.q.device

    def to(self, device) -> "FP8Weight":
        return FP8Weight(self.q.to(device), self.sf.to(device))

    def dequant(self) -> torch.Tensor:
        N, Kd = self.q.shape
        s = torch.pow(2.0, self.sf.float() - 127.0)
        s = s.repeat_interleave(GROUP, 0)[:N].repeat_interleave(GROUP, 1)
        return self.q.float() * s

    def rows(self, lo: int, hi: int) -> "FP8Weight":
        """Rows [lo, hi) of the weight (lo, hi multiples of 128)."""
        assert lo % GROUP == 0 and (hi % GROUP == 0 or hi == self.q.shape[0])
        return FP8Weight(self.q[lo:hi].contiguous(), self.sf[lo // GROUP:-(-hi // GROUP)].contiguous())

    def cols(self, lo: int, hi: int) -> "FP8Weight":
        """Columns (K) [lo, hi) of the weight (multiples of 128)."""
        assert lo % GROUP == 0 and hi % GROUP == 0
        return FP8Weight(self.q[:, lo:hi].contiguous(), self.sf[:, lo // GROUP:hi // GROUP].contiguous())


def _exp_pow2(amax: torch.Tensor) -> torch.Tensor:
    """Smallest integer e with amax / 2^e <= 448, clamped to [-126, 126];
    0 where amax == 0."""
    r = amax.float() / E4M3_MAX
    m, ex = torch.frexp(r)  # r = m * 2^ex, m in [0.5, 1)
    e = torch.where(m == 0.5, ex - 1, ex)
    e = torch.where(r > 0, e, torch.zeros_like(e))
    return e.clamp(-126, 126).to(torch.int32)


def quantize_weight(w: torch.Tensor) -> FP8Weight:
    """[N, K] float weight -> e4m3 with one power-of-two scale per 128x128
    block (K must be a multiple of 128)."""
    N, Kd = w.shape
    if Kd % GROUP:
        raise ValueError(f"K={Kd} is not a multiple of {GROUP}")
    nb = -(-N // GROUP)
    wp = torch.zeros(nb * GROUP, Kd, dtype=torch.float32, device=w.device)
    wp[:N] = w.float()
    blocks = wp.view(nb, GROUP, Kd // GROUP, GROUP)
    e = _exp_pow2(blocks.abs().amax(dim=(1, 3)))
    inv = torch.pow(2.0, -e.float())[:, None, :, None]
    q = (blocks * inv).view(nb * GROUP, Kd)[:N].to(torch.float8_e4m3fn)
    return FP8Weight(q.contiguous(), (e + 127).to(torch.uint8))


def random_weight(N: int, Kd: int, std: float, generator: torch.Generator | None = None,
                  device: str | torch.device = "cpu") -> FP8Weight:
    w = torch.randn(N, Kd, generator=generator) * std
    return quantize_weight(w).to(device)


def quant_act(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (e4m3 [M, K], uint8 scales [K/128, M])."""
    M, Kd = x.shape
    if Kd % GROUP:
        raise ValueError(f"K={Kd} is not a multiple of {GROUP}")
    if not x.is_cuda:
        g = x.float().view(M, Kd // GROUP, GROUP)
        e = _exp_pow2(g.abs().amax(dim=2))
        q = (g * torch.pow(2.0, -e.float())[:, :, None]).view(M, Kd).to(torch.float8_e4m3fn)
        return q, (e + 127).to(torch.uint8).t().contiguous()
    assert x.dtype == torch.bfloat16 and x.stride(1) == 1
    q = torch.empty(M, Kd, dtype=torch.float8_e4m3fn, device=x.device)
    sf = torch.empty(Kd // GROUP, max(M, 1), dtype=torch.uint8, device=x.device)
    rc = _native.kernels().ib_quant_fp8_act(x.data_ptr(), x.stride(0), M, Kd, q.data_ptr(), q.stride(0),
                                            sf.data_ptr(), sf.stride(0), K._stream())
    _native.check(rc, "ib_quant_fp8_act")
    K._count(1)
    return q, sf


def dequant_act(q: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    M, Kd = q.shape
    s = torch.pow(2.0, sf[:, :M].float() - 127.0).t().repeat_interleave(GROUP, 1)
    return q.float() * s


_fp8_plan_cache: dict[tuple[int, int, int], int] = {}


def _splits(M: int, N: int, Kd: int) -> int:
    key = (M, N, Kd)
    s = _fp8_plan_cache.get(key)
    if s is None:
        out = (_native.c_int * 7)()
        _native.kernels().ib_gemm_fp8_plan(M, N, Kd, K._num_sms(), 0, out)
        s = _fp8_plan_cache[key] = int(out[4])
    return s


def gemm_fp8(q: torch.Tensor, sf: torch.Tensor, w: FP8Weight, out: torch.Tensor | None = None,
             swiglu: bool = False) -> torch.Tensor:
    """bf16 [M, N] (N/2 with ``swiglu``) = dequant(q, sf) @ dequant(w)^T,
    fp32 accumulation."""
    M, Kd = q.shape
    N = w.q.shape[0]
    n_out = N // 2 if swiglu else N
    if not q.is_cuda:
        y = dequant_act(q, sf) @ w.dequant().t()
        if swiglu:
            y = torch.nn.functional.silu(y[:, 0::2]) * y[:, 1::2]
        y = y.to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(M, n_out, dtype=torch.bfloat16, device=q.device)
    sc = K.scratch(q.device)
    splits = _splits(M, N, Kd)
    ws = sc.ensure_gemm(M * N if splits > 1 else 1)
    rc = _native.kernels().ib_gemm_fp8(q.data_ptr(), sf.data_ptr(), sf.stride(0), w.q.data_ptr(), w.sf.data_ptr(),
                                       out.data_ptr(), M, N, Kd, q.stride(0), w.q.stride(0), out.stride(0),
                                       1 if swiglu else 0, ws.data_ptr(), 0, sc.status.data_ptr(), K._stream())
    _native.check(rc, "ib_gemm_fp8")
    K._count(2 if splits > 1 and not K._FUSED_REDUCE else 1)
    return out


def linear(x: torch.Tensor, w: FP8Weight, out: torch.Tensor | None = None, swiglu: bool = False) -> torch.Tensor:
    """bf16 activations through an fp8 weight: quantise, then block-scaled GEMM."""
    q, sf = quant_act(x)
    return gemm_fp8(q, sf, w, out=out, swiglu=swiglu)


def gemm_fp8_grouped(xp: torch.Tensor, w: FP8Weight, n_experts: int, offsets: torch.Tensor, swiglu: bool = False,
                     bn: int | None = None) -> torch.Tensor:
    """Grouped fp8 GEMM over experts: rows of ``xp`` [R, K] (bf16, sorted by
    expert, ``offsets`` [E+1]) times their expert's block of ``w`` (the E
    experts' [N, K] weights stacked to [E*N, K])."""
    R, Kd = xp.shape
    N = w.q.shape[0] // n_experts
    n_out = N // 2 if swiglu else N
    if not xp.is_cuda:
        wd = w.dequant().view(n_experts, N, Kd)
        q, sf = quant_act(xp)
        xd = dequant_act(q, sf)
        y = torch.zeros(R, N, dtype=torch.float32)
        off = offsets.tolist()
        for e in range(n_experts):
            a, b = off[e], off[e + 1]
            if b > a:
                y[a:b] = xd[a:b] @ wd[e].t()
        if swiglu:
            y = torch.nn.functional.silu(y[:, 0::2]) * y[:, 1::2]
        return y.to(torch.bfloat16)
    q, sf = quant_act(xp)
    out = torch.empty(R, n_out, dtype=torch.bfloat16, device=xp.device)
    bn = bn or K.grouped_bn(R, n_experts)
    bn = min(192, max(32, ((bn + 31) // 32) * 32))  # the fp8 kernel's token tiles: multiples of 32, <= 192
    cap = (-(-R // bn) + n_experts) * (N // 128)
    tab = torch.empty(cap * 4 + 1, dtype=torch.int32, device=xp.device)
    num = tab[cap * 4:]
    lib = _native.kernels()
    _native.check(lib.ib_moe_tiles(offsets.data_ptr(), n_experts, N, bn, tab.data_ptr(), num.data_ptr(), K._stream()),
                  "ib_moe_tiles")
    sc = K.scratch(xp.device)
    rc = lib.ib_gemm_fp8_grouped(q.data_ptr(), sf.data_ptr(), sf.stride(0), w.q.data_ptr(), w.sf.data_ptr(),
                                 out.data_ptr(), R, N, Kd, n_experts, q.stride(0), w.q.stride(0), out.stride(0),
                                 1 if swiglu else 0, tab.data_ptr(), num.data_ptr(), bn, cap, sc.status.data_ptr(),
                                 K._stream())
    _native.check(rc, "ib_gemm_fp8_grouped")
    K._count(2)
    return out

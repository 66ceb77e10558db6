"""Mixture-of-experts FFN on the sm_100a kernels (DeepSeek-V3 shape).

    logits  = x @ Wg^T                         tcgen05 GEMM (bf16)
    ids, w  = grouped top-k(sigmoid(logits) + bias)   ib_moe_topk
    rows    = sort (token, slot) pairs by expert        ib_moe_permute
    xp      = x[token_of_row]                            gather
    act     = silu(xp We_gate^T) * (xp We_up^T)          grouped GEMM, SwiGLU epilogue
    out_r   = act @ We_down^T                            grouped GEMM
    y       = sum_j w[t, j] * out_r[row(t, j)]           ib_moe_combine
    y      += shared expert (dense SwiGLU MLP) when configured

Weights are random-initialised from a seed like the dense model's. The
routing can be passed in (``ids`` / ``wts``) so a test can hold it fixed.
"""

from __future__ import annotations

import math

import torch

from infera_b200.ops import kernels as K


class MoELayer:
    def __init__(self, hidden: int, moe_ffn: int, num_experts: int, top_k: int, n_groups: int = 1,
                 topk_groups: int = 1, routed_scaling: float = 1.0, num_shared: int = 0,
                 device: str | torch.device = "cuda", seed: int = 0, std: float = 0.02, weight_dtype: str = "bf16",
                 expert_range: tuple[int, int] | None = None):
        """``expert_range=(lo, hi)``: build only experts lo..hi-1 (an expert-
        parallel shard; the router still scores all ``num_experts``). Each
        expert's weights come from its own seed, so a shard holds exactly
        the rows the full layer would."""
        self.H, self.F, self.E, self.k = hidden, moe_ffn, num_experts, top_k
        self.n_groups, self.topk_groups, self.scaling = n_groups, topk_groups, routed_scaling
        self.lo, self.hi = expert_range if expert_range is not None else (0, num_experts)
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        bf = torch.bfloat16

        def rnd(*shape, scale=std, gen=g):
            return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * scale).to(bf)

        self.gate = rnd(num_experts, hidden, scale=1.0 / math.sqrt(hidden))
        self.bias = torch.zeros(num_experts, dtype=torch.float32, device=dev)
        n = self.hi - self.lo
        self.w13 = torch.empty(n, 2 * moe_ffn, hidden, dtype=bf, device=dev)   # interleaved gate / up rows
        self.w2 = torch.empty(n, hidden, moe_ffn, dtype=bf, device=dev)
        for e in range(self.lo, self.hi):
            ge = torch.Generator(device=dev).manual_seed(seed * 1_000_003 + 7 * e + 1)
            self.w13[e - self.lo] = rnd(2 * moe_ffn, hidden, gen=ge)
            self.w2[e - self.lo] = rnd(hidden, moe_ffn, scale=std / math.sqrt(2), gen=ge)
        self.shared = None
        if num_shared:
            self.shared = (rnd(2 * moe_ffn * num_shared, hidden), rnd(hidden, moe_ffn * num_shared))
        # fp8: experts stacked to [n*2F, H] / [n*H, F] e4m3 with 128x128 block scales
        self.fp8 = weight_dtype == "fp8"
        if self.fp8:
            from infera_b200.ops import fp8

            self.w13 = fp8.quantize_weight(self.w13.reshape(n * 2 * moe_ffn, hidden))
            self.w2 = fp8.quantize_weight(self.w2.reshape(n * hidden, moe_ffn))
            if self.shared is not None:
                self.shared = tuple(fp8.quantize_weight(t) for t in self.shared)

    def route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        logits = K.linear(x, self.gate)
        return K.moe_topk(logits, self.k, self.n_groups, self.topk_groups, self.bias, self.scaling)

    def forward(self, x: torch.Tensor, ids: torch.Tensor | None = None, wts: torch.Tensor | None = None
                ) -> torch.Tensor:
        if ids is None:
            ids, wts = self.route(x)
        offsets, row_of_slot, token_of_row = K.moe_permute(ids, self.E)
        xp = K.gather_rows(x, token_of_row)
        if self.fp8:
            from infera_b200.ops import fp8

            act = fp8.gemm_fp8_grouped(xp, self.w13, self.E, offsets, swiglu=True)
            rows = fp8.gemm_fp8_grouped(act, self.w2, self.E, offsets)
        else:
            act = K.gemm_grouped(xp, self.w13, offsets, swiglu=True)
            rows = K.gemm_grouped(act, self.w2, offsets)
        y = K.moe_combine(rows, row_of_slot, wts)
        if self.shared is not None:
            y = y + K.linear(K.linear(x, self.shared[0], swiglu=True), self.shared[1])
        return y

    def expert(self, e: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Expert e's (w13 [2F, H], w2 [H, F]) as fp32 (dequantised if fp8)."""
        if self.fp8:
            return (self.w13.rows(e * 2 * self.F, (e + 1) * 2 * self.F).dequant(),
                    self.w2.rows(e * self.H, (e + 1) * self.H).dequant())
        return self.w13[e].float(), self.w2[e].float()

    def to(self, device) -> "MoELayer":
        for name in ("gate", "bias", "w13", "w2"):
            setattr(self, name, getattr(self, name).to(device))
        if self.shared is not None:
            self.shared = tuple(t.to(device) for t in self.shared)
        return self

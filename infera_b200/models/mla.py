"""DeepSeek-V3-shaped decoder: multi-head latent attention (MLA) + routed
experts, over a paged cache of 576-wide latent rows.

Per layer (q_lora_rank > 0):

    x       = rmsnorm(h)
    q       = q_b(rmsnorm(q_a(x)))                [T, Hq, nope 128 | rope 64]
    kva     = kv_a(x)                             [T, kv_lora 512 | rope 64]
    q_lat   = W_UK[h] q_nope[h]   per head        [T, Hq, 512]     (absorbed)
    cache   = [rmsnorm(kva[:512]) | rope(kva[512:])]  at each token's slot
    o_lat   = MQA(q = [q_lat | rope(q_pe)], K = cache, V = cache[:, :512])
    attn    = W_UV[h] o_lat[h]    per head        [T, Hq * 128]
    h      += o(attn);  x = rmsnorm(h)
    h      += FFN(x)   dense SwiGLU for the first layers, routed experts
                       (+ shared expert) after

The per-head absorptions run as grouped GEMMs with the heads as groups
(``ib_gemm_grouped``), decode tokens' attention as ``ib_mla_decode`` (each
token a query with its own causal key count). Prompt chunks take the
non-absorbed path: every sequence's latent context is up-projected once to
per-head [k_nope | v] (one GEMM against ``w_kv_up``) and attended by the
flash-attention kernel over 128 + 64 score dims with 128-dim values, which
needs no W_UV absorption afterwards (``M.mla_prefill``; the absorbed decode
kernel for prompt tokens too when ``INFERA_MLA_PREFILL=absorbed``). The big
projections run as fp8 block-scaled GEMMs when ``weight_dtype`` is "fp8". RoPE rotates pairs (i, i + 32) of the 64 rope dims (a fixed
permutation of the interleaved pairing of the published checkpoints; the
weights here are random).

Reference counterpart: the DeepSeek-V3 EP=8 configuration the reference
serves through SGLang / vLLM (``examples/`` recipes); the model code lives in
those engines, not in the reference tree.
"""

from __future__ import annotations

import math

import torch

from infera_b200.models.config import MoEConfig
from infera_b200.models.dense import ForwardBatch
from infera_b200.ops import kernels as K
from infera_b200.ops import mla as M


class MLAWeights:
    def __init__(self, cfg: MoEConfig, device: torch.device, seed: int = 0, std: float = 0.02,
                 expert_range: tuple[int, int] | None = None):
        """``expert_range``: routed experts built per MoE layer (an expert-
        parallel rank's shard; None: all)."""
        self.cfg = cfg
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        fp8 = cfg.weight_dtype == "fp8"
        if fp8:
            from infera_b200.ops import fp8 as F8

        def rnd(*shape, scale=std):
            return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * scale).to(bf)

        def lin(*shape, scale=std):
            w = rnd(*shape, scale=scale)
            return F8.quantize_weight(w) if fp8 else w

        H, Hq = cfg.hidden, cfg.num_heads
        dn, dr, dv, L = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
        self.embed = rnd(cfg.vocab, H, scale=1.0)
        out_scale = std / math.sqrt(2 * cfg.num_layers)
        self.layers = []
        for li in range(cfg.num_layers):
            lw = {"ln1": torch.ones(H, dtype=bf, device=device), "ln2": torch.ones(H, dtype=bf, device=device)}
            if cfg.q_lora_rank > 0:
                lw["q_a"] = lin(cfg.q_lora_rank, H)
                lw["q_a_norm"] = torch.ones(cfg.q_lora_rank, dtype=bf, device=device)
                lw["q_b"] = lin(Hq * (dn + dr), cfg.q_lora_rank)
            else:
                lw["q"] = lin(Hq * (dn + dr), H)
            lw["kv_a"] = lin(L + dr, H)
            lw["kv_a_norm"] = torch.ones(L, dtype=bf, device=device)
            # kv_b split per head: W_UK [Hq, L, dn] (q_lat = W_UK q_nope) and
            # W_UV [Hq, dv, L] (out = W_UV o_lat), both K-major for the GEMMs
            lw["w_uk"] = rnd(Hq, L, dn, scale=1.0 / math.sqrt(dn))
            lw["w_uv"] = rnd(Hq, dv, L, scale=1.0 / math.sqrt(L))
            lw["w_kv_up"] = M.kv_up_weight(lw["w_uk"], lw["w_uv"])
            lw["o"] = lin(H, Hq * dv, scale=out_scale)
            if cfg.is_moe_layer(li):
                from infera_b200.models.moe import MoELayer

                lw["moe"] = MoELayer(H, cfg.moe_ffn, cfg.num_experts, cfg.top_k, cfg.n_groups, cfg.topk_groups,
                                     cfg.routed_scaling, cfg.num_shared_experts, device, seed=seed * 1000 + li,
                                     std=std, weight_dtype=cfg.weight_dtype, expert_range=expert_range)
            else:
                lw["gate_up"] = lin(2 * cfg.dense_ffn, H)
                lw["down"] = lin(H, cfg.dense_ffn, scale=out_scale)
            self.layers.append(lw)
        self.final_norm = torch.ones(H, dtype=bf, device=device)
        self.lm_head = rnd(cfg.vocab, H)

    def nbytes(self) -> int:
        n = 2 * (self.embed.numel() + self.lm_head.numel() + self.final_norm.numel())
        for lw in self.layers:
            for k, t in lw.items():
                if k == "moe":
                    for w in (t.w13, t.w2, *(t.shared or ())):
                        n += w.q.numel() + w.sf.numel() if not isinstance(w, torch.Tensor) else 2 * w.numel()
                    n += 2 * t.gate.numel()
                elif isinstance(t, torch.Tensor):
                    n += 2 * t.numel()
                else:
                    n += t.q.numel() + t.sf.numel()
        return n


class MLAModel:
    """Stateless forward over the paged latent cache owned by the engine
    (``k_caches`` [num_layers, slots, 576]; ``v_caches`` is unused)."""

    prefill_tile_rows = 128   # the 192-dim prefill attention runs one query tile per CTA

    def __init__(self, cfg: MoEConfig, device: torch.device | str, seed: int = 0, tp=None, ep=None):
        """``ep``: expert parallelism under data-parallel attention - an
        object with ``rank``, ``world``, ``group`` (the all-to-all group),
        ``gloo`` and ``fused``; every MoE layer keeps only this rank's
        E / world experts and exchanges tokens with the other ranks."""
        if tp is not None and tp.world > 1:
            raise NotImplementedError("tensor parallelism of MLA layers (use data-parallel attention + EP)")
        self.full_cfg = cfg
        self.cfg = cfg
        self.tp = None
        self.device = torch.device(device)
        shard = None
        if ep is not None and ep.world > 1:
            el = cfg.num_experts // ep.world
            shard = (ep.rank * el, (ep.rank + 1) * el)
        self.w = MLAWeights(cfg, self.device, seed=seed, expert_range=shard)
        self.ep = ep
        if ep is not None and ep.world > 1:
            from infera_b200.parallel.ep import EPMoE

            for lw in self.w.layers:
                if "moe" in lw:
                    lw["moe"] = EPMoE(lw["moe"], ep.rank, ep.world, group=ep.group, device=self.device,
                                      fused=ep.fused, max_tokens=ep.max_tokens, gloo_group=ep.gloo)
        self.cos_sin = K.rope_cos_sin(cfg.max_model_len, cfg.qk_rope_dim, cfg.rope_theta, None, device=self.device)
        self.scale = M.default_scale(cfg.qk_nope_dim, cfg.qk_rope_dim)
        import os

        # the kernel takes 128 nope + 64 rope score dims and 128 value dims;
        # the CPU restatement takes any
        self.prefill_unabsorbed = (os.environ.get("INFERA_MLA_PREFILL", "flash") != "absorbed"
                                   and (self.device.type == "cpu" or (cfg.qk_nope_dim == 128 and cfg.v_head_dim == 128
                                                                      and cfg.qk_rope_dim == 64)))

    def _query_meta(self, fb: ForwardBatch, T: int) -> tuple[torch.Tensor, torch.Tensor, int]:
        """Per-token block-table row, visible key count and the largest one."""
        Tp = fb.num_prefill_tokens
        parts = []
        max_len = 0
        if Tp > 0:
            q_len, ctx_len = fb.p_host_meta
            rows = fb.p_bt_rows if fb.p_bt_rows is not None else torch.arange(len(q_len), device=self.device,
                                                                               dtype=torch.int32)
            lens = torch.tensor(q_len, device=self.device)
            parts.append(torch.repeat_interleave(rows, lens, output_size=Tp))
            max_len = max(ctx_len)
        if fb.num_decode > 0:
            parts.append(fb.d_bt_rows if fb.d_bt_rows is not None else
                         torch.arange(fb.num_decode, device=self.device, dtype=torch.int32))
            max_len = max(max_len, 8192 if self.device.type == "cuda" else 0)
        q_row = parts[0] if len(parts) == 1 else torch.cat(parts)
        q_kvlen = (fb.positions[:T] + 1).to(torch.int32)
        return q_row.to(torch.int32), q_kvlen, max_len

    def _absorb(self, x_hm: torch.Tensor, w: torch.Tensor, T: int) -> torch.Tensor:
        Hq = self.cfg.num_heads
        offsets = torch.arange(Hq + 1, device=x_hm.device, dtype=torch.int32) * T
        return K.gemm_grouped(x_hm, w, offsets)

    def forward(self, fb: ForwardBatch, k_caches: torch.Tensor, v_caches: torch.Tensor | None = None,
                bufs: dict | None = None) -> torch.Tensor:
        cfg = self.cfg
        T = fb.token_ids.shape[0]
        H, Hq = cfg.hidden, cfg.num_heads
        dn, dr, dv, L = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
        bufs = bufs or {}
        h = K.embed(fb.token_ids, self.w.embed, out=bufs["h"][:T] if "h" in bufs else None)
        x = K.rmsnorm(h, self.w.layers[0]["ln1"], cfg.rms_eps)
        q_row, q_kvlen, max_len = self._query_meta(fb, T)
        bt = fb.p_block_table if fb.num_prefill_tokens > 0 else fb.d_block_table
        Tp = fb.num_prefill_tokens
        pf = self.prefill_unabsorbed and Tp > 0      # prompt rows take the non-absorbed path
        T0 = Tp if pf else 0                          # first row that is absorbed
        Ta = T - T0
        for li, lw in enumerate(self.w.layers):
            if "q_a" in lw:
                qa = K.rmsnorm(K.linear(x, lw["q_a"]), lw["q_a_norm"], cfg.rms_eps)
                qb = K.linear(qa, lw["q_b"])
            else:
                qb = K.linear(x, lw["q"])
            kva = K.linear(x, lw["kv_a"])
            qb3 = qb.view(T, Hq, dn + dr)
            q_full = torch.empty(T, Hq, L + dr, dtype=torch.bfloat16, device=self.device)
            if Ta > 0:
                q_nope_hm = qb3[T0:, :, :dn].transpose(0, 1).contiguous().view(Hq * Ta, dn)
                q_lat = self._absorb(q_nope_hm, lw["w_uk"], Ta).view(Hq, Ta, L)
                q_full[T0:, :, :L] = q_lat.transpose(0, 1)
            q_full[:, :, L:] = qb3[:, :, dn:]
            cache = k_caches[li]
            M.mla_rope_kvwrite(q_full, kva, fb.positions, fb.slots, self.cos_sin, lw["kv_a_norm"], cfg.rms_eps,
                               cache)
            if fb.layer_hook is not None:
                fb.layer_hook(li)   # this layer's latent rows are written (layer-by-layer KV push)
            attn = torch.empty(T, Hq * dv, dtype=torch.bfloat16, device=self.device)
            if pf:
                M.mla_prefill(qb[:Tp], q_full[:Tp], cache, fb.p_block_table, fb.p_bt_rows, fb.p_host_meta,
                              fb.p_q_start, fb.p_q_len, fb.p_ctx_len, fb.p_tiles, lw["w_kv_up"], Hq, dn, dv,
                              self.scale, out=attn[:Tp], dr=dr)
            if Ta > 0:
                o_lat = M.mla_attention(q_full[T0:], cache, bt, q_row[T0:], q_kvlen[T0:], self.scale,
                                        max_kvlen=max_len, rope_dim=dr)
                o_hm = o_lat.transpose(0, 1).contiguous().view(Hq * Ta, L)
                attn[T0:] = self._absorb(o_hm, lw["w_uv"], Ta).view(Hq, Ta, dv).transpose(0, 1).reshape(Ta, Hq * dv)
            o = K.linear(attn, lw["o"])
            x = K.add_rmsnorm(o, h, lw["ln2"], cfg.rms_eps, out=torch.empty_like(x))
            if "moe" in lw:
                y = lw["moe"].forward(x)
            else:
                y = K.linear(K.linear(x, lw["gate_up"], swiglu=True), lw["down"])
            nxt = self.w.layers[li + 1]["ln1"] if li + 1 < cfg.num_layers else self.w.final_norm
            x = K.add_rmsnorm(y, h, nxt, cfg.rms_eps, out=torch.empty_like(x))
        xs = K.gather_rows(x, fb.logits_idx)
        return K.linear(xs, self.w.lm_head, out=bufs["logits"][: xs.shape[0]] if "logits" in bufs else None)

    def alloc_buffers(self, max_tokens: int, max_seqs: int) -> dict:
        bf = torch.bfloat16
        return {"h": torch.empty(max_tokens, self.cfg.hidden, dtype=bf, device=self.device),
                "logits": torch.empty(max_seqs, self.cfg.vocab, dtype=bf, device=self.device)}

    def max_gemm_workspace(self, max_tokens: int) -> int:
        cfg = self.cfg
        return max_tokens * max(cfg.num_heads * cfg.head_dim, 2 * cfg.dense_ffn, cfg.vocab)


def reference_logits_mla(model: MLAModel, token_ids: list[int]) -> torch.Tensor:
    """Plain fp32 forward of the MLA decoder on the CPU, NOT absorbed:
    per-head keys k = [W_UK^T c | k_pe] and values v = W_UV c expanded from
    the latent, standard causal attention. fp8 projections quantise their
    inputs the way the engine does."""
    from infera_b200.models.reference import _moe_ref

    cfg = model.cfg
    w = model.w
    T = len(token_ids)
    Hq, dn, dr, dv, L = cfg.num_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
    ids = torch.tensor(token_ids, dtype=torch.long)
    cs = model.cos_sin.cpu()[:T]
    cos, sin = cs[..., 0], cs[..., 1]

    def f(t):
        return t.detach().float().cpu()

    def mm(x, wt):
        if isinstance(wt, torch.Tensor):
            return x @ f(wt).t()
        from infera_b200.ops import fp8

        q, sf = fp8.quant_act(x.to(torch.bfloat16))
        return fp8.dequant_act(q, sf) @ wt.to("cpu").dequant().t()

    def norm(x, g):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * f(g)

    def rope(x):  # [T, ..., dr]
        half = dr // 2
        a, b = x[..., :half], x[..., half:]
        shape = (T,) + (1,) * (x.dim() - 2) + (half,)
        c, s = cos.view(shape), sin.view(shape)
        return torch.cat([a * c - b * s, b * c + a * s], dim=-1)

    h = f(w.embed)[ids]
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    for lw in w.layers:
        x = norm(h, lw["ln1"])
        qb = mm(norm(mm(x, lw["q_a"]), lw["q_a_norm"]), lw["q_b"]) if "q_a" in lw else mm(x, lw["q"])
        qb = qb.view(T, Hq, dn + dr)
        kva = mm(x, lw["kv_a"])
        c = norm(kva[:, :L], lw["kv_a_norm"])
        k_pe = rope(kva[:, L:])                                      # [T, dr]
        q_pe = rope(qb[:, :, dn:])                                   # [T, Hq, dr]
        wuk, wuv = f(lw["w_uk"]), f(lw["w_uv"])                      # [Hq, L, dn], [Hq, dv, L]
        k_nope = torch.einsum("tl,hld->thd", c, wuk)                 # [T, Hq, dn]
        v = torch.einsum("tl,hvl->thv", c, wuv)                      # [T, Hq, dv]
        s = (torch.einsum("thd,shd->hts", qb[:, :, :dn], k_nope)
             + torch.einsum("thd,sd->hts", q_pe, k_pe)) * model.scale
        s = s.masked_fill(mask[None], float("-inf"))
        o = torch.einsum("hts,shv->thv", torch.softmax(s, -1), v).reshape(T, Hq * dv)
        h = h + mm(o, lw["o"])
        x = norm(h, lw["ln2"])
        if "moe" in lw:
            h = h + _moe_ref(lw["moe"], x, f)
        else:
            gu = mm(x, lw["gate_up"])
            h = h + mm(torch.nn.functional.silu(gu[:, 0::2]) * gu[:, 1::2], lw["down"])
    return norm(h, w.final_norm) @ f(w.lm_head).t()

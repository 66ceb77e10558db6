"""Dense GQA decoder (Llama-3 / Qwen3 shapes) on the sm_100a ops.

The forward pass works on a flat batch of tokens (``ForwardBatch``): first
the prefill chunks of zero or more sequences, then one token for each
decoding sequence. Per layer:

    qkv  = x @ Wqkv^T                       tcgen05 GEMM
    rope(q, k); k, v -> paged cache         fused kernel
    attn = prefill FA (chunks) | decode split-KV (one token per seq)
    o    = attn @ Wo^T                      tcgen05 GEMM
    h   += o ; x = rmsnorm(h)               fused kernel
    act  = silu(x Wg^T) * (x Wu^T)          tcgen05 GEMM, SwiGLU epilogue
    d    = act @ Wd^T                       tcgen05 GEMM
    h   += d ; x = rmsnorm(h)               fused kernel (next layer's norm)

The gate/up weight is stored row-interleaved (gate_0, up_0, gate_1, ...)
so the GEMM epilogue can apply SwiGLU without a second pass.
Only the rows in ``logits_idx`` reach the LM head.

Tensor parallelism (``tp``: a :class:`infera_b200.parallel.comm.TPComm`):
QKV and gate/up are column-parallel (each rank owns 1/world of the heads
and of the MLP width), the attention output and MLP down projections are
row-parallel and each is followed by an all-reduce fused with the residual
add and the next RMSNorm (NVLink one-shot push for small batches, NCCL
otherwise); the LM head is vocab-parallel and its logits are all-gathered
(fused into the LM-head GEMM's epilogue, which stores each rank's column
block into every rank's logits over NVLink, up to the batch the symmetric
buffer holds; NCCL otherwise).
``model.cfg`` is this rank's local shape; ``model.full_cfg`` the model's.
Weights are generated full-size from the seed and sliced, so any TP size
computes the same model.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from infera_b200.models.config import DenseConfig
from infera_b200.ops import kernels as K


@dataclass
class ForwardBatch:
    """Device-side metadata of one engine step (all int32 on the model's device)."""

    token_ids: torch.Tensor        # [T]
    positions: torch.Tensor        # [T]
    slots: torch.Tensor            # [T] cache slot of each token (page*16+off)
    logits_idx: torch.Tensor       # [S] rows whose logits are needed
    num_prefill_tokens: int = 0
    # prefill (chunks) metadata
    p_q_start: torch.Tensor | None = None
    p_q_len: torch.Tensor | None = None
    p_ctx_len: torch.Tensor | None = None
    p_block_table: torch.Tensor | None = None
    p_tiles: torch.Tensor | None = None
    p_host_meta: tuple[list[int], list[int]] | None = None
    p_bt_rows: torch.Tensor | None = None
    # decode metadata (rows [num_prefill_tokens, T))
    d_block_table: torch.Tensor | None = None
    d_seq_lens: torch.Tensor | None = None
    d_bt_rows: torch.Tensor | None = None
    d_splits: int = 1
    d_tps: int = 0                 # decode attention tiles per split (0: even split)
    num_decode: int = 0
    layer_hook: object = None  # called with the layer index after its KV write


class DenseWeights:
    def __init__(self, cfg: DenseConfig, device: torch.device, seed: int = 0, std: float = 0.02,
                 rank: int = 0, world: int = 1):
        self.cfg = cfg
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def rnd(*shape, scale=std):
            return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * scale).to(bf)

        H, D, W, r = cfg.hidden, cfg.head_dim, world, rank
        hq, hk = cfg.num_heads // W, cfg.num_kv_heads // W
        f = cfg.ffn // W
        q_rows = slice(r * hq * D, (r + 1) * hq * D)
        k_rows = slice(cfg.q_size + r * hk * D, cfg.q_size + (r + 1) * hk * D)
        v_rows = slice(cfg.q_size + cfg.kv_size + r * hk * D, cfg.q_size + cfg.kv_size + (r + 1) * hk * D)

        def shard_rows(t, *sl):
            return t if W == 1 else torch.cat([t[x] for x in sl], 0).contiguous()

        def shard_cols(t, a, b):
            return t if W == 1 else t[:, a:b].contiguous()

        self.embed = rnd(cfg.vocab, H, scale=1.0)
        self.layers = []
        out_scale = std / math.sqrt(2 * cfg.num_layers)
        for li in range(cfg.num_layers):
            qkv = rnd(cfg.qkv_size, H)
            o = rnd(H, cfg.q_size, scale=out_scale)
            gu = rnd(2 * cfg.ffn, H)      # interleaved rows (g0, u0, g1, u1, ...)
            dn = rnd(H, cfg.ffn, scale=out_scale)
            lw = {
                "ln1": torch.ones(H, dtype=bf, device=device),
                "ln2": torch.ones(H, dtype=bf, device=device),
                "qkv": shard_rows(qkv, q_rows, k_rows, v_rows),
                "o": shard_cols(o, r * hq * D, (r + 1) * hq * D),
                "gate_up": shard_rows(gu, slice(2 * r * f, 2 * (r + 1) * f)),
                "down": shard_cols(dn, r * f, (r + 1) * f),
            }
            del qkv, o, gu, dn
            if cfg.weight_dtype == "fp8":
                from infera_b200.ops import fp8

                for key in ("qkv", "o", "gate_up", "down"):
                    lw[key] = fp8.quantize_weight(lw[key])
            if cfg.is_moe_layer(li):
                if W > 1:
                    raise NotImplementedError("tensor parallelism of expert layers (use expert parallelism)")
                from infera_b200.models.moe import MoELayer

                del lw["gate_up"], lw["down"]
                lw["moe"] = MoELayer(H, cfg.moe_ffn, cfg.num_experts, cfg.moe_top_k, cfg.moe_n_groups,
                                     cfg.moe_topk_groups, cfg.moe_routed_scaling, cfg.moe_num_shared, device,
                                     seed=seed * 1000 + li, std=std)
            if cfg.qk_norm:
                lw["q_norm"] = torch.ones(cfg.head_dim, dtype=bf, device=device)
                lw["k_norm"] = torch.ones(cfg.head_dim, dtype=bf, device=device)
            self.layers.append(lw)
        self.final_norm = torch.ones(H, dtype=bf, device=device)
        lm = rnd(cfg.vocab, H)
        vl = cfg.vocab // W
        self.lm_head = lm if W == 1 else lm[r * vl:(r + 1) * vl].contiguous()
        del lm

    def nbytes(self) -> int:
        n = 2 * (self.embed.numel() + self.lm_head.numel() + self.final_norm.numel())
        for lw in self.layers:
            for k, t in lw.items():
                if k == "moe":
                    n += 2 * (t.w13.numel() + t.w2.numel() + t.gate.numel())
                elif isinstance(t, torch.Tensor):
                    n += 2 * t.numel()
                else:  # fp8 weight: 1 byte per element + one scale byte per block
                    n += t.q.numel() + t.sf.numel()
        return n


class DenseModel:
    """Stateless forward over a paged KV cache owned by the engine."""

    def __init__(self, cfg: DenseConfig, device: torch.device | str, seed: int = 0, tp=None):
        self.full_cfg = cfg
        self.tp = tp
        W = tp.world if tp is not None else 1
        r = tp.rank if tp is not None else 0
        if cfg.num_heads % W or cfg.num_kv_heads % W or cfg.ffn % W or cfg.vocab % W:
            raise ValueError(f"{cfg.name} does not split over {W} tensor-parallel ranks")
        self.cfg = replace(cfg, num_heads=cfg.num_heads // W, num_kv_heads=cfg.num_kv_heads // W,
                           ffn=cfg.ffn // W) if W > 1 else cfg
        self.device = torch.device(device)
        self.w = DenseWeights(cfg, self.device, seed=seed, rank=r, world=W)
        self.cos_sin = K.rope_cos_sin(cfg.max_model_len, cfg.head_dim, cfg.rope_theta, cfg.rope_scaling,
                                      device=self.device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    # ------------------------------------------------------------------
    def _qk_norm(self, qkv: torch.Tensor, lw: dict) -> None:
        cfg = self.cfg
        T = qkv.shape[0]
        D = cfg.head_dim
        nq, nk = cfg.num_heads, cfg.num_kv_heads
        q = qkv[:, : nq * D].reshape(T * nq, D)
        k = qkv[:, nq * D:(nq + nk) * D].reshape(T * nk, D)
        qkv[:, : nq * D] = K.rmsnorm(q.contiguous(), lw["q_norm"], cfg.rms_eps).view(T, nq * D)
        qkv[:, nq * D:(nq + nk) * D] = K.rmsnorm(k.contiguous(), lw["k_norm"], cfg.rms_eps).view(T, nk * D)

    def forward(self, fb: ForwardBatch, k_caches: torch.Tensor, v_caches: torch.Tensor,
                bufs: dict | None = None) -> torch.Tensor:
        """Returns logits [S, vocab] for the rows in ``fb.logits_idx``.

        ``k_caches`` / ``v_caches``: [num_layers, num_slots, kv_size] bf16.
        ``bufs``: optional preallocated activations (used by CUDA graphs).
        """
        cfg = self.cfg
        T = fb.token_ids.shape[0]
        Tp = fb.num_prefill_tokens
        H = cfg.hidden
        dev = self.device
        bf = torch.bfloat16
        if bufs is None:
            bufs = {}
        h = bufs.get("h")
        h = K.embed(fb.token_ids, self.w.embed, out=None if h is None else h[:T])
        x = bufs["x"][:T] if "x" in bufs else torch.empty(T, H, dtype=bf, device=dev)
        qkv = bufs["qkv"][:T] if "qkv" in bufs else torch.empty(T, cfg.qkv_size, dtype=bf, device=dev)
        attn = bufs["attn"][:T] if "attn" in bufs else torch.empty(T, cfg.q_size, dtype=bf, device=dev)
        o = bufs["o"][:T] if "o" in bufs else torch.empty(T, H, dtype=bf, device=dev)
        act = bufs["act"][:T] if "act" in bufs else torch.empty(T, cfg.ffn, dtype=bf, device=dev)
        K.rmsnorm(h, self.w.layers[0]["ln1"], cfg.rms_eps, out=x)
        for li, lw in enumerate(self.w.layers):
            kc, vc = k_caches[li], v_caches[li]
            # a split qkv GEMM hands its fp32 workspace to rope_kvwrite (no
            # finalize launch); with q / k norms the finalized rows are needed
            ws = None if cfg.qk_norm else K.linear_deferred(x, lw["qkv"], qkv)
            if ws is not None:
                K.rope_kvwrite_ws(ws, qkv, fb.positions, fb.slots, self.cos_sin, cfg.num_heads, cfg.num_kv_heads,
                                  cfg.head_dim, kc, vc)
            else:
                if cfg.qk_norm:
                    K.linear(x, lw["qkv"], out=qkv)
                    self._qk_norm(qkv, lw)
                K.rope_kvwrite(qkv, fb.positions, fb.slots, self.cos_sin, cfg.num_heads, cfg.num_kv_heads,
                               cfg.head_dim, kc, vc)
            if fb.layer_hook is not None:
                fb.layer_hook(li)
            if Tp > 0:
                K.attn_prefill(qkv[:Tp], kc, vc, fb.p_block_table, fb.p_q_start, fb.p_q_len, fb.p_ctx_len,
                               fb.p_tiles, cfg.num_heads, cfg.num_kv_heads, self.scale, out=attn[:Tp],
                               host_meta=fb.p_host_meta, bt_rows=fb.p_bt_rows)
            if fb.num_decode > 0:
                K.attn_decode(qkv[Tp:T], kc, vc, fb.d_block_table, fb.d_seq_lens, cfg.num_heads, cfg.num_kv_heads,
                              self.scale, splits=fb.d_splits, out=attn[Tp:T], bt_rows=fb.d_bt_rows,
                              tiles_per_split=fb.d_tps)
            nxt = self.w.layers[li + 1]["ln1"] if li + 1 < cfg.num_layers else self.w.final_norm
            if "moe" in lw:
                K.linear(attn, lw["o"], out=o)
                K.add_rmsnorm(o, h, lw["ln2"], cfg.rms_eps, out=x)
                y = lw["moe"].forward(x)
                K.add_rmsnorm(y, h, nxt, cfg.rms_eps, out=x)
            elif self.tp is None:
                # split o / down GEMMs hand their fp32 workspace to add_rmsnorm
                ws = K.linear_deferred(attn, lw["o"], o)
                if ws is None:
                    K.add_rmsnorm(o, h, lw["ln2"], cfg.rms_eps, out=x)
                else:
                    K.add_rmsnorm_ws(ws, h, lw["ln2"], cfg.rms_eps, out=x)
                K.linear(x, lw["gate_up"], out=act, swiglu=True)
                ws = K.linear_deferred(act, lw["down"], o)
                if ws is None:
                    K.add_rmsnorm(o, h, nxt, cfg.rms_eps, out=x)
                else:
                    K.add_rmsnorm_ws(ws, h, nxt, cfg.rms_eps, out=x)
            else:
                self.tp.gemm_allreduce_add_rmsnorm(attn, lw["o"], h, lw["ln2"], cfg.rms_eps, x, 0, tmp=o)
                K.linear(x, lw["gate_up"], out=act, swiglu=True)
                self.tp.gemm_allreduce_add_rmsnorm(act, lw["down"], h, nxt, cfg.rms_eps, x, 1, tmp=o)
        S = fb.logits_idx.shape[0]
        xs = bufs["xs"][:S] if "xs" in bufs else None
        xs = K.gather_rows(x, fb.logits_idx, out=xs)
        logits = bufs["logits"][:S] if "logits" in bufs else None
        if self.tp is None or self.tp.world == 1:
            return K.linear(xs, self.w.lm_head, out=logits)
        fused = getattr(self.tp, "uses_fused_gather", None)
        if fused is not None and fused(S, self.w.lm_head.shape[0], self.w.lm_head):
            # vocab-parallel LM head with the all-gather fused into its epilogue
            return self.tp.gemm_allgather_cols(xs, self.w.lm_head)
        local = K.linear(xs, self.w.lm_head, out=bufs["logits_local"][:S] if "logits_local" in bufs else None)
        return self.tp.all_gather_cols(local, out=logits)

    def alloc_buffers(self, max_tokens: int, max_seqs: int) -> dict:
        cfg = self.cfg
        bf = torch.bfloat16
        dev = self.device
        if self.tp is not None and self.tp.world > 1 and hasattr(self.tp, "ensure_gather"):
            self.tp.ensure_gather(max_seqs, self.full_cfg.vocab)
        return {
            "h": torch.empty(max_tokens, cfg.hidden, dtype=bf, device=dev),
            "x": torch.empty(max_tokens, cfg.hidden, dtype=bf, device=dev),
            "qkv": torch.empty(max_tokens, cfg.qkv_size, dtype=bf, device=dev),
            "attn": torch.empty(max_tokens, cfg.q_size, dtype=bf, device=dev),
            "o": torch.empty(max_tokens, cfg.hidden, dtype=bf, device=dev),
            "act": torch.empty(max_tokens, cfg.ffn, dtype=bf, device=dev),
            "xs": torch.empty(max_seqs, cfg.hidden, dtype=bf, device=dev),
            "logits": torch.empty(max_seqs, cfg.vocab, dtype=bf, device=dev),
            **({"logits_local": torch.empty(max_seqs, self.w.lm_head.shape[0], dtype=bf, device=dev)}
               if self.tp is not None and self.tp.world > 1 else {}),
        }

    def max_gemm_workspace(self, max_tokens: int) -> int:
        cfg = self.cfg
        widest = max(cfg.qkv_size, cfg.hidden, 2 * cfg.ffn, cfg.vocab)
        return max_tokens * widest

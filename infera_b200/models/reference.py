"""Plain fp32 PyTorch forward of the dense decoder over a full sequence
(no paging, no chunking, no cache). The oracle for engine tests."""

from __future__ import annotations

import torch

from infera_b200.models.dense import DenseModel


@torch.no_grad()
def reference_logits(model: DenseModel, token_ids: list[int]) -> torch.Tensor:
    """Logits [len(token_ids), vocab] in fp32, computed on the CPU."""
    cfg = model.cfg
    w = model.w
    T = len(token_ids)
    D = cfg.head_dim
    nq, nk = cfg.num_heads, cfg.num_kv_heads
    G = nq // nk
    ids = torch.tensor(token_ids, dtype=torch.long)
    cs = model.cos_sin.cpu()[:T]
    cos, sin = cs[..., 0], cs[..., 1]

    def f(t):
        return t.detach().float().cpu()

    def mm(x, wt):
        """x @ W^T; an fp8 weight also quantises x the way the engine does
        (e4m3 with a power-of-two scale per token and 128-wide group)."""
        if isinstance(wt, torch.Tensor):
            return x @ f(wt).t()
        from infera_b200.ops import fp8

        q, sf = fp8.quant_act(x.to(torch.bfloat16))
        return fp8.dequant_act(q, sf) @ wt.to("cpu").dequant().t()

    def norm(x, g, eps=cfg.rms_eps):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * f(g)

    def rope(x):  # [T, heads, D]
        half = D // 2
        a, b = x[..., :half], x[..., half:]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat([a * c - b * s, b * c + a * s], dim=-1)

    h = f(w.embed)[ids]
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    for lw in w.layers:
        x = norm(h, lw["ln1"])
        qkv = mm(x, lw["qkv"])
        q = qkv[:, : nq * D].view(T, nq, D)
        k = qkv[:, nq * D:(nq + nk) * D].view(T, nk, D)
        v = qkv[:, (nq + nk) * D:].view(T, nk, D)
        if cfg.qk_norm:
            q = norm(q, lw["q_norm"])
            k = norm(k, lw["k_norm"])
        q, k = rope(q), rope(k)
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        s = torch.einsum("thd,shd->hts", q, k) / D ** 0.5
        s = s.masked_fill(mask[None], float("-inf"))
        o = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, nq * D)
        h = h + mm(o, lw["o"])
        x = norm(h, lw["ln2"])
        if "moe" in lw:
            h = h + _moe_ref(lw["moe"], x, f)
            continue
        gu = mm(x, lw["gate_up"])
        act = torch.nn.functional.silu(gu[:, 0::2]) * gu[:, 1::2]
        h = h + mm(act, lw["down"])
    x = norm(h, w.final_norm)
    return x @ f(w.lm_head).t()


def _moe_ref(m, x: torch.Tensor, f) -> torch.Tensor:
    """fp32 routed experts (+ shared): the same grouped routing as the kernels."""
    from infera_b200.ops import kernels as K

    logits = x @ f(m.gate).t()
    ids, wts = K.moe_topk(logits, m.k, m.n_groups, m.topk_groups, f(m.bias), m.scaling)

    def qa(v):  # activations as the fp8 kernels see them
        if not m.fp8:
            return v
        from infera_b200.ops import fp8

        q, sf = fp8.quant_act(v.reshape(-1, v.shape[-1]).to(torch.bfloat16))
        return fp8.dequant_act(q, sf).reshape(v.shape)

    def wt(t):
        return t.to("cpu").dequant() if not isinstance(t, torch.Tensor) else f(t)

    y = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(m.k):
            w13, w2 = (w.cpu() for w in m.expert(int(ids[t, j])))
            gu = qa(x[t:t + 1]) @ w13.t()
            a = torch.nn.functional.silu(gu[:, 0::2]) * gu[:, 1::2]
            y[t] += float(wts[t, j]) * (qa(a) @ w2.t())[0]
    if m.shared is not None:
        gu = qa(x) @ wt(m.shared[0]).t()
        y += qa(torch.nn.functional.silu(gu[:, 0::2]) * gu[:, 1::2]) @ wt(m.shared[1]).t()
    return y


def reference_greedy(model: DenseModel, prompt: list[int], n: int) -> tuple[list[int], list[float]]:
    """Greedy continuation and the top1-top2 logit margin at each step."""
    toks = list(prompt)
    out, margins = [], []
    for _ in range(n):
        lg = reference_logits(model, toks)[-1]
        top = torch.topk(lg, 2)
        out.append(int(top.indices[0]))
        margins.append(float(top.values[0] - top.values[1]))
        toks.append(out[-1])
    return out, margins
